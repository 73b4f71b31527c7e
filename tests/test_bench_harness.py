"""CPU checks of bench.py's config-4 harness (the BoltModel-shaped decoder).

The decoder's cached-key/value path (one prefill step, then one-token steps) must give the
same logits as a plain forward over the whole sequence, so that the tok/s the bench reports
are those of a correct model.  Runs in float32 on the CPU: no GPU, no libebx.
"""
from __future__ import annotations

import sys
from pathlib import Path

import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def test_bolt_shape_matches_baseline_config4():
    c = bench.BOLT
    assert (c["vocab"], c["dim"], c["heads"], c["kv_heads"], c["layers"], c["ffn_mult"]) == \
        (32000, 384, 12, 1, 6, 4)
    assert (c["batch"], c["prefill"], c["steps"]) == (8, 512, 128)


def test_bolt_incremental_decode_equals_full_forward():
    torch.manual_seed(0)
    m = bench._bolt_model("cpu").float()
    assert m.lm_head.weight is m.embed.weight  # tied output head (kept FP16 by ElasticBit)
    ids = torch.randint(0, bench.BOLT["vocab"], (2, 12))
    caches = [(k.float(), v.float()) for k, v in m.new_caches(2, "cpu")]
    with torch.no_grad():
        logits = m.step(ids, caches, torch.arange(12))
        toks = [logits.argmax(-1, keepdim=True)]
        outs = []
        for t in range(3):
            outs.append(m.step(toks[-1], caches, torch.tensor([12 + t])))
            toks.append(outs[-1].argmax(-1, keepdim=True))
        for t in range(3):
            seq = torch.cat([ids] + toks[:t + 1], dim=1)
            fresh = [(k.float(), v.float()) for k, v in m.new_caches(2, "cpu")]
            ref = m.step(seq, fresh, torch.arange(seq.shape[1]))
            assert torch.allclose(outs[t], ref, rtol=1e-4, atol=1e-5), (t, (outs[t] - ref).abs().max())

"""ElasticBit parity checker (test infrastructure; never imported by the product)."""

"""CPU oracle for the kvcache path (test infrastructure; never imported by the product).

See ``oracle/kv_oracle.py`` for the restated reference algorithms.
"""

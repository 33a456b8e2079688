"""kvcache operator modules of the B200 backend."""

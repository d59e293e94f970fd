"""Magic Transformer: a research toy (MoD routing, cross-layer KV reuse, dual streams, router feedback)."""

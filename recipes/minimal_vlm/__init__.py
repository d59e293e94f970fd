"""Minimal VLM example: Qwen3-VL SFT without packing (one padded row per sample)."""

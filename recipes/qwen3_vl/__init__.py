"""Qwen3-VL full-SFT recipe."""

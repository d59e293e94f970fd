"""Qwen3 dense-decoder text pretraining recipe."""

"""OpenBee: three-stage Qwen3-VL training (projector alignment, full SFT, long-image SFT with spike guard)."""

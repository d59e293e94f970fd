"""B200 data plane: native flat FSDP, fused optimizer, context / tensor parallel runtimes."""

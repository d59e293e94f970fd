from .collator import MinimalVLMCollator
from .dataset import build_dataset
from .preprocess import build_sample_spec, process_sample
from .processor import build_qwen3_vl_processor

__all__ = ["MinimalVLMCollator", "build_dataset", "build_qwen3_vl_processor", "build_sample_spec", "process_sample"]

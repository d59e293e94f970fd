from .collator import MinimalVLMCollator
from .dataset import build_dataset
from .preprocess import build_sample_spec, convert_images_to_pixel_values, process_image, process_sample
from .processor import build_qwen3_vl_processor

__all__ = ["MinimalVLMCollator", "build_dataset", "build_qwen3_vl_processor", "build_sample_spec",
           "convert_images_to_pixel_values", "process_image", "process_sample"]

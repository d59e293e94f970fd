from .media import QwenImageHandler, QwenVLMediaHandler, read_image
from .processor import QwenVLImageProcessor, QwenVLProcessor, smart_resize
from .schema import QwenVLChatSchemaHandler
from ..tokenization import QwenVLTokenizationHandler

__all__ = ["QwenImageHandler", "QwenVLMediaHandler", "read_image", "QwenVLImageProcessor", "QwenVLProcessor",
           "smart_resize", "QwenVLChatSchemaHandler", "QwenVLTokenizationHandler"]

from .schema import QwenChatSchemaHandler
from .tokenization import QwenChatTokenizationHandler

__all__ = ["QwenChatSchemaHandler", "QwenChatTokenizationHandler"]

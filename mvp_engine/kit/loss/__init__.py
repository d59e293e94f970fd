from .loss import LossGuard, LossKit
from .token_loss import PerTokenLossGuard, TokenLossStats, TokenNormedLossKit, apply_chunked_token_loss_patch

__all__ = ["LossGuard", "LossKit", "PerTokenLossGuard", "TokenLossStats", "TokenNormedLossKit",
           "apply_chunked_token_loss_patch"]

from .detokenize import DetokenizeManager, printable_prefix
from .server import tokenize_worker
from .tokenize import TokenizeManager

__all__ = ["DetokenizeManager", "TokenizeManager", "printable_prefix", "tokenize_worker"]

from .layout import TPLayout
from .state import TPState, get_tp, init_tp, set_tp

__all__ = ["TPLayout", "TPState", "get_tp", "init_tp", "set_tp"]

from .AdamW_adv import AdamW_adv
from .Lion_adv import Lion_adv
from .Prodigy_adv import Prodigy_adv

__all__ = ["AdamW_adv", "Lion_adv", "Prodigy_adv"]

from .AdamW_adv import AdamW_adv

__all__ = ["AdamW_adv"]

from .AdaMuon_adv import AdaMuon_adv
from .AdamW_adv import AdamW_adv
from .Lion_adv import Lion_adv
from .Muon_adv import Muon_adv
from .Prodigy_adv import Prodigy_adv
from ._muon_family import newton_schulz

__all__ = ["AdamW_adv", "Lion_adv", "Prodigy_adv", "Muon_adv", "AdaMuon_adv", "newton_schulz"]

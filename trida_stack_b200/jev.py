"""Compatibility names of the decision ("jev") data and loss (the reference's ``train.jev``,
deprecated there); use ``trida_stack_b200.data.decision`` / ``trida_stack_b200.models.decision``."""
import warnings

from .data.decision import DecisionRowDataset as JevRowDataset  # noqa: F401
from .data.decision import load_decision_records as load_jev_records  # noqa: F401
from .data.decision import pack_decision as pack_jev  # noqa: F401
from .models.decision import PointerHead  # noqa: F401
from .models.decision import decision_loss as jev_loss  # noqa: F401

warnings.warn("trida_stack_b200.jev is a compatibility name; use trida_stack_b200.data.decision and "
              "trida_stack_b200.models.decision", DeprecationWarning, stacklevel=2)

"""Compatibility import of the decision head, loss and row encoder under one name (the
reference's ``train.decision``, deprecated there)."""
from .data.decision import encode_rows, materialize, pack_decision  # noqa: F401
from .models.decision import PointerHead, decision_loss  # noqa: F401

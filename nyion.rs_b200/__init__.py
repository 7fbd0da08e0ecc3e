"""nyion.rs_b200 — B200-native attention hot path of bmcc-DEV/Nyion.rs.

The product is the C-ABI library ``libnyion_attn.so`` (sources in ``csrc/``,
ABI in ``include/nyion_attn.h``).  ``attn`` binds it for Python callers with
torch tensors as device buffers.
"""
from . import attn  # noqa: F401

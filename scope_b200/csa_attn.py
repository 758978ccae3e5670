"""Drop-in for the reference's `csa_attn_kernel` module
(kernel/cpu_attn_ds4_ext/csa_attn.cpp:1885-1977), on CUDA tensors."""
from __future__ import annotations

from .cpu_attn import get_num_threads, set_num_threads  # noqa: F401  (same no-op semantics)

"""KV byte accounting used by admission and by the prefix-cache budget.

Restates ContinuousBatchingEngine._kv_bytes_per_token
(src/mlxz/engine/continuous.py:170-178) and AdmissionController._project_peak
(src/mlxz/scheduler/admission.py:98-104): 2 (K and V) * layers * KV heads *
head_dim * bits / 8 bytes per token (the engine's ``_n_heads`` is the KV head
count, continuous.py:103-107), and the peak of a request as (prompt + max new
tokens) times that.  Scale and bias bytes of quantised KV are not in the
reference's formula; ``store_bytes_per_token`` gives the exact bytes a paged
store of this package holds per token.
"""
from __future__ import annotations

from typing import Any


def kv_bytes_per_token(n_layers: int, n_kv_heads: int, head_dim: int, bits: int) -> float:
    """2 * n_layers * n_kv_heads * head_dim * bits / 8 (continuous.py:170-178)."""
    return 2 * n_layers * n_kv_heads * head_dim * (bits / 8)


def project_peak(prompt_tokens: int, max_new_tokens: int, n_layers: int, n_kv_heads: int,
                 head_dim: int, bits: int) -> int:
    """Peak KV bytes of a request (admission.py:98-104)."""
    total = prompt_tokens + max_new_tokens
    return int(total * kv_bytes_per_token(n_layers, n_kv_heads, head_dim, bits))


def store_bytes_per_token(store: Any) -> int:
    """Bytes a paged store holds per token over all layers, K and V (codes,
    scales and biases for a quantised store)."""
    return int(store.bytes_per_token)

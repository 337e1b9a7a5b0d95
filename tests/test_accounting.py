"""KV byte accounting (continuous.py:170-178, admission.py:98-104)."""
import pytest

from mlxz_b200.engine.accounting import kv_bytes_per_token, project_peak


@pytest.mark.parametrize("L,H,D,bits,want", [
    (32, 8, 128, 16, 131072.0),   # 8B shape, bf16: 2 * 32 * 8 * 128 * 2
    (32, 8, 128, 8, 65536.0),
    (32, 8, 128, 4, 32768.0),
    (80, 8, 128, 16, 327680.0),   # 70B shape
    (16, 8, 64, 16, 32768.0),     # 1B shape
])
def test_kv_bytes_per_token(L, H, D, bits, want):
    assert kv_bytes_per_token(L, H, D, bits) == want


def test_project_peak_rounds_down_like_the_reference():
    assert project_peak(100, 28, 32, 8, 128, 16) == 128 * 131072
    # fractional bytes per token (bits not a multiple of 8) truncate with int()
    assert project_peak(3, 0, 1, 1, 3, 4) == int(3 * 2 * 1 * 1 * 3 * 0.5)
    assert project_peak(0, 0, 32, 8, 128, 8) == 0

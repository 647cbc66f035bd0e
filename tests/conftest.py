import pathlib
import sys

import numpy as np
import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100a GPU (B200); run with -m gpu")


@pytest.fixture(scope="session")
def ctx():
    from shardlm_b200.runtime import Context

    c = Context(0)
    yield c
    c.close()


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle

    return oracle


def bf16_round(a: np.ndarray) -> np.ndarray:
    """Round f32 to the nearest bf16 (ties to even); returns the uint16 bit patterns."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint32) << 16).view(np.float32)


def f32_sum_tolerance(k: int, abs_sum: np.ndarray) -> np.ndarray:
    """Bound on |a - b| for two f32 summations of the same k products in different orders.

    Each order is within gamma_k * sum|x_i w_i| of the exact value (Higham, Accuracy and Stability
    of Numerical Algorithms, thm 3.1 with gamma_k = k u / (1 - k u), u = 2^-24), so two orders
    differ by at most 2 gamma_k sum|x_i w_i|.
    """
    u = 2.0 ** -24
    gamma = k * u / (1 - k * u)
    return 2.0 * gamma * abs_sum + 1e-30

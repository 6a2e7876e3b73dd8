"""Host-side checks of the batched evaluation search (no GPU needed)."""

import math

import pytest


def test_options_follow_the_reference_checks():
    # mcts/src/PUCT.cpp:161-175
    from kingdom_ai import PUCTOptions
    PUCTOptions()
    for kwargs, message in (
            (dict(simulations=0), "at least one simulation"),
            (dict(simulations=True), "at least one simulation"),
            (dict(c_puct=0.0), "exploration coefficient"),
            (dict(c_puct=math.inf), "exploration coefficient"),
            (dict(dirichlet_alpha=-1.0), "Dirichlet alpha"),
            (dict(dirichlet_epsilon=1.5), "Dirichlet epsilon"),
            (dict(dirichlet_epsilon=math.nan), "Dirichlet epsilon"),
            (dict(c_puct=True), "real numbers"),
            (dict(time_limit_ms=-1), "unsigned"),
            (dict(seed=2**64), "unsigned")):
        with pytest.raises(ValueError, match=message):
            PUCTOptions(**kwargs)


def test_searcher_needs_a_cuda_device():
    from kingdom_ai import GpuBatchedPUCT
    with pytest.raises((ValueError, RuntimeError)):
        GpuBatchedPUCT(4, device="cpu")


def test_workspace_size_is_computable_on_cpu():
    import ctypes
    from kingdom_ai import _native as native
    lib = native.library()
    fn = lib.gk_bpuct_workspace_bytes
    fn.argtypes = [ctypes.c_int64, ctypes.c_int, ctypes.c_int]
    fn.restype = ctypes.c_size_t
    small, large = fn(4, 100, 8), fn(4, 200, 8)
    assert 0 < small < large
    assert fn(0, 100, 8) == 0 and fn(4, 0, 8) == 0 and fn(4, 100, 0) == 0
    per_node_edges = 82 * (8 + 8 + 4 + 4 + 4)
    assert large - small >= 4 * 100 * per_node_edges

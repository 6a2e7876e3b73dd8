"""gk_puct_search_hash_noalloc (static device scratch) against gk_puct_search_hash.

The allocation-free entry point keeps its search trees in one device array
that every call reuses, so each call has to reproduce the workspace entry
point exactly even though the previous call left the array dirty: two calls
in a row with different batch sizes, depths and options are compared field
by field. Requests above the array's size are refused with GK_ENOSPC before
anything is launched. The file sorts last so the array is also exercised in
a process where all the other GPU tests have run; it passes on its own too.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

GK_EINVAL = -22
GK_ENOSPC = -28
SCRATCH_BYTES = 16 * 1024 * 1024  # GK_NOALLOC_SCRATCH_BYTES
FIELDS = ("actions", "visits", "policy", "values", "simulations", "evaluations", "priors", "best_values", "nodes",
          "root_values", "status")


def _noalloc_fn():
    from kingdom_ai import _native as native

    return native.register("gk_puct_search_hash_noalloc",
                           [ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(native.PuctOptions),
                            ctypes.POINTER(native.PuctResults), ctypes.c_void_p])


def _roots(n, seed):
    from kingdom_ai import _native as native

    bits = torch.empty((n, 16), dtype=torch.int32, device="cuda")
    native.call("gk_gen_positions", seed, 0, n, native.ptr(bits), native.stream_of(bits.device))
    return bits


def _options(c_puct=1.5, epsilon=0.0, fpu=None):
    from kingdom_ai import _native as native

    return native.PuctOptions(float(c_puct), float(epsilon), 0 if fpu is None else 1, float(fpu or 0.0))


def _with_workspace(roots, sims, opts):
    """The existing entry point on a fresh caller workspace."""
    from kingdom_ai import _native as native
    from kingdom_ai.gpu_puct import SearchWorkspace, _allocate_results

    n = roots.shape[0]
    ws = SearchWorkspace(n, sims + 1, roots.device)
    out = _allocate_results(n, roots.device)
    native.call("gk_puct_search_hash", ws.pointer, n, sims, native.ptr(roots), opts, out.struct,
                native.stream_of(roots.device))
    torch.cuda.synchronize()
    return out


def _noalloc(roots, sims, opts):
    from kingdom_ai import _native as native
    from kingdom_ai.gpu_puct import _allocate_results

    n = roots.shape[0]
    out = _allocate_results(n, roots.device)
    rc = _noalloc_fn()(n, sims, native.ptr(roots), opts, out.struct, native.stream_of(roots.device))
    torch.cuda.synchronize()
    return rc, out


def _assert_same(got, want):
    for name in FIELDS:
        assert torch.equal(getattr(got, name), getattr(want, name)), name


def test_two_calls_in_a_row_match_the_workspace_entry_point():
    first_roots, second_roots = _roots(48, 101), _roots(20, 202)
    first_opts, second_opts = _options(1.5), _options(1.25, fpu=0.2)
    rc1, first = _noalloc(first_roots, 40, first_opts)
    rc2, second = _noalloc(second_roots, 64, second_opts)
    assert (rc1, rc2) == (0, 0)
    _assert_same(first, _with_workspace(first_roots, 40, first_opts))
    _assert_same(second, _with_workspace(second_roots, 64, second_opts))
    # Non-trivial searches: every live root ran all its simulations.
    assert int(first.simulations.max()) == 40 and int(second.simulations.max()) == 64
    assert int(first.status.item()) == 0 and int(second.status.item()) == 0


def test_a_dirty_scratch_gives_the_same_results():
    """20 trees of 400 simulations fill the array; 256 trees of 28 then run
    over bytes the first search left behind and must still equal the
    workspace entry point."""
    assert _noalloc(_roots(20, 303), 400, _options())[0] == 0
    roots = _roots(256, 304)
    opts = _options(c_puct=1.25)
    rc, got = _noalloc(roots, 28, opts)
    assert rc == 0
    _assert_same(got, _with_workspace(roots, 28, opts))


def test_largest_request_runs_and_a_larger_one_is_refused():
    from kingdom_ai import _native as native

    lib = native.library()
    assert lib.gk_puct_workspace_bytes(20, 401) <= SCRATCH_BYTES < lib.gk_puct_workspace_bytes(21, 401)
    roots = _roots(20, 405)
    rc, got = _noalloc(roots, 400, _options())
    assert rc == 0
    _assert_same(got, _with_workspace(roots, 400, _options()))
    rc, refused = _noalloc(_roots(21, 406), 400, _options())
    assert rc == GK_ENOSPC
    assert bool((refused.actions == -1).all()) and int(refused.visits.abs().sum()) == 0


def test_invalid_arguments_are_rejected():
    from kingdom_ai import _native as native
    from kingdom_ai.gpu_puct import _allocate_results

    fn = _noalloc_fn()
    roots = _roots(4, 7)
    out = _allocate_results(4, roots.device)
    stream = native.stream_of(roots.device)
    assert fn(0, 8, native.ptr(roots), _options(), out.struct, stream) == GK_EINVAL
    assert fn(4, 0, native.ptr(roots), _options(), out.struct, stream) == GK_EINVAL
    assert fn(4, 8, None, _options(), out.struct, stream) == GK_EINVAL
    assert fn(4, 8, native.ptr(roots), None, out.struct, stream) == GK_EINVAL
    # This search draws no root noise, so a noise weight is refused.
    assert fn(4, 8, native.ptr(roots), _options(epsilon=0.25), out.struct, stream) == GK_EINVAL
    # Sizes whose byte counts would overflow are refused before any arithmetic.
    assert fn(1 << 62, 8, native.ptr(roots), _options(), out.struct, stream) == GK_ENOSPC
    assert fn(4, 2**31 - 1, native.ptr(roots), _options(), out.struct, stream) == GK_ENOSPC

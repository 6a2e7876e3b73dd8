"""The C ABI library loads and exports every symbol include/gk.h declares (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("gk*.h"))
LIBRARY = ROOT / "alpha-yoo-for-great-kingdom_b200" / "kingdom_ai" / "libgk.so"


def declared_symbols():
    names = []
    for header in HEADERS:
        names += re.findall(r"^GK_API\s+[\w\s\*]*?\b(gk_\w+)\s*\(", header.read_text(), flags=re.M)
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert len(names) >= 30
    assert len(names) == len(set(names))
    assert "gk_timer_create" in names and "gk_selfplay_ply" in names


def test_every_declaration_has_its_own_comment():
    for header in HEADERS:
        lines = header.read_text().splitlines()
        for i, line in enumerate(lines):
            if line.startswith("GK_API"):
                above = lines[i - 1].strip()
                assert above.endswith("*/"), f"{header.name}:{i + 1} {line}"


def test_library_exports_every_declared_symbol():
    if not LIBRARY.exists():
        pytest.skip("libgk.so not built")
    lib = ctypes.CDLL(str(LIBRARY))
    missing = [name for name in declared_symbols() if not hasattr(lib, name)]
    assert not missing, f"not exported: {missing}"


def test_every_declaration_cites_a_reference_interface_or_says_it_has_none():
    for header in HEADERS:
        text = header.read_text()
        for match in re.finditer(r"(/\*(?:(?!\*/).)*\*/)\s*GK_API[^;]*?(gk_\w+)\s*\(", text, flags=re.S):
            comment, name = match.group(1), match.group(2)
            assert ("Replaces" in comment or "replaces" in comment or "reference" in comment
                    or ".py:" in comment or ".cpp:" in comment or "Equivalent" in comment
                    or "Same" in comment or "workspace" in comment or "stands in" in comment), name


def test_workspace_size_is_computable_on_cpu():
    if not LIBRARY.exists():
        pytest.skip("libgk.so not built")
    lib = ctypes.CDLL(str(LIBRARY))
    fn = lib.gk_puct_workspace_bytes
    fn.argtypes = [ctypes.c_int64, ctypes.c_int]
    fn.restype = ctypes.c_size_t
    small = fn(4, 9)
    assert small > 4 * 9 * 82 * 24
    assert fn(0, 9) == 0 and fn(4, 0) == 0
    # 4096 trees x 401 nodes fit comfortably in 180 GB of HBM.
    assert fn(4096, 401) < 8 * 1024**3


def test_search_options_validation_matches_reference():
    from kingdom_ai.gpu_puct import GpuPUCTOptions

    # python/kingdom_ai/gpu_puct.py:26-63 and tests/gpu_puct_test.py:44-55
    assert GpuPUCTOptions().tactical_checks is False
    assert GpuPUCTOptions().fpu_reduction is None
    for value in (0, 1, None, "true"):
        with pytest.raises(TypeError):
            GpuPUCTOptions(tactical_checks=value)
    for value in (True, -1, float("nan"), float("inf"), "0"):
        with pytest.raises(ValueError):
            GpuPUCTOptions(fpu_reduction=value)
    for value in (0, 0.1, 0.25):
        assert GpuPUCTOptions(fpu_reduction=value).fpu_reduction == value
    for bad in (dict(simulations=0), dict(c_puct=0), dict(dirichlet_alpha=-1), dict(dirichlet_epsilon=1.5),
                dict(seed=-1), dict(seed=2**64), dict(c_puct=float("nan"))):
        with pytest.raises(ValueError):
            GpuPUCTOptions(**bad)


def test_product_never_imports_the_oracle():
    package = ROOT / "alpha-yoo-for-great-kingdom_b200"
    for path in list(package.rglob("*.py")) + list(package.rglob("*.cu")) + list(package.rglob("*.cuh")):
        text = path.read_text()
        assert "oracle" not in text.replace("the oracle", ""), path


def test_collect_gpu_puct_games_validates_like_the_reference():
    """python/kingdom_ai/gpu_training.py:150-168; all checks run before any device work."""
    from kingdom_ai.gpu_puct import HashEvaluator
    from kingdom_ai.training import collect_gpu_puct_games

    assert collect_gpu_puct_games(HashEvaluator(), 0) == []
    for kw, exc in (({"games": -1}, ValueError), ({"batch_size": 0}, ValueError), ({"seed": -1}, ValueError),
                    ({"temperature": float("nan")}, ValueError), ({"temperature": True}, TypeError),
                    ({"temperature_moves": -2}, ValueError), ({"record_history": 1}, TypeError),
                    ({"options": object()}, TypeError)):
        args = {"games": 1, **kw}
        games = args.pop("games")
        with pytest.raises(exc):
            collect_gpu_puct_games(HashEvaluator(), games, **args)


def test_network_pointers_must_be_16_byte_aligned():
    """gk_net_forward refuses a network whose bulk-copied arrays are not
    16-byte aligned before it touches the GPU (the pointers are never read)."""
    if not LIBRARY.exists():
        pytest.skip("libgk.so not built")
    from kingdom_ai._native import NetStruct

    lib = ctypes.CDLL(str(LIBRARY))
    fn = lib.gk_net_forward
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    base = 1 << 20
    names = ["conv_w", "conv_b", "head_w", "head_b", "pol_w", "pol_b", "val_w1", "val_b1", "val_w2", "val_b2"]
    for bad in ("conv_w", "conv_b", "pol_w", "val_w1"):
        net = NetStruct()
        net.channels, net.blocks, net.norm = 64, 6, 0
        for k, name in enumerate(names):
            setattr(net, name, base + 4096 * k + (4 if name == bad else 0))
        rc = fn(ctypes.byref(net), base, None, 8, base, base, base, base, None)
        assert rc == -22, bad

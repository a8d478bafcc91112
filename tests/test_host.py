"""Host-side logic of the product (no GPU): schedule / routing / compile against the reference's
goldens and invariants, the C ABI's exported symbols and argument validation, and the rule that
there is no CPU fallback."""
import ctypes
import math
import os
import re

import pytest
import torch

from conftest import REPO


# ---------------------------------------------------------------- wavefront host logic
def verify_schedule(grid_shape, deps, schedule):
    """Completeness, no duplicates, every dependency strictly earlier
    (wavefront/wavefront_test.py:10-48)."""
    seen = {}
    for t, group in enumerate(schedule):
        for c in group:
            assert c not in seen, f"duplicate {c}"
            seen[c] = t
    assert len(seen) == math.prod(grid_shape)
    for c, t in seen.items():
        for off, _ in deps:
            d = tuple(a + b for a, b in zip(c, off))
            if all(0 <= d[i] < grid_shape[i] for i in range(len(c))):
                assert seen[d] < t
    return True


def test_schedule_matches_reference(wf_golden):
    from wavefront import WavefrontConfig, generate_wavefront_schedule
    c2 = WavefrontConfig(grid_shape=(4, 4), batch_size=1)
    c3 = WavefrontConfig(grid_shape=(3, 8, 8), batch_size=1,
                         dependencies=[((-1, 0, 0), 0), ((0, -1, 0), 1), ((0, 0, -1), 1)])
    cf = WavefrontConfig(grid_shape=(4, 6), batch_size=1,
                         dependencies=[((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)], num_ports=4)
    for cfg, key in ((c2, "schedule_4x4"), (c3, "schedule_3x8x8"), (cf, "schedule_flb_4x6")):
        s = generate_wavefront_schedule(cfg)
        assert s == wf_golden[key]
        assert verify_schedule(cfg.grid_shape, cfg.dependencies, s)


def test_schedule_long_chain_no_recursion_limit():
    """The FLB model's grid (12 x 1024, three dependencies) has 2058 ticks."""
    from wavefront import WavefrontConfig, generate_wavefront_schedule
    cfg = WavefrontConfig(grid_shape=(12, 1024), batch_size=1,
                          dependencies=[((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)], num_ports=4)
    s = generate_wavefront_schedule(cfg)
    assert len(s) == 2058
    assert max(len(g) for g in s) == 6
    # a pure-left chain: 5000 cells in one row, each depending on its left neighbour
    cfg2 = WavefrontConfig(grid_shape=(1, 5000), batch_size=1, dependencies=[((0, -1), 0)],
                           num_ports=1)
    s2 = generate_wavefront_schedule(cfg2)
    assert len(s2) == 5000


def test_engine_routing_and_compile(wf_golden):
    import torch.nn as nn
    from wavefront import WavefrontConfig, WavefrontEngine
    cfg = WavefrontConfig(grid_shape=(3, 4), batch_size=2, dim=8)
    eng = WavefrontEngine(cfg, nn.ModuleList([nn.Identity() for _ in range(3)]))
    assert torch.equal(eng.routing_map, wf_golden["routing_3x4"])
    assert (eng.compiled_cells, eng.compiled_layers, eng.max_cells_per_tick) == \
        tuple(wf_golden["compiled_3x4"])
    cf = WavefrontConfig(grid_shape=(4, 6), batch_size=1,
                         dependencies=[((-1, 0), 0), ((0, -1), 1), ((1, -1), 2)], num_ports=4)
    ef = WavefrontEngine(cf, nn.ModuleList([nn.Identity() for _ in range(4)]))
    assert torch.equal(ef.routing_map, wf_golden["routing_flb_4x6"])
    assert (ef.compiled_cells, ef.compiled_layers, ef.max_cells_per_tick) == \
        tuple(wf_golden["compiled_flb_4x6"])


def test_mapped_fetcher_kat():
    """Known answer of wavefront/wavefront_test.py:147-184: cell (1,2) = flat 6 reads flat 2 on
    port 0 (dep (-1,0)) and flat 5 on port 1 (dep (0,-1))."""
    import torch.nn as nn
    from wavefront import WavefrontConfig, WavefrontEngine, fetch_mapped_context
    cfg = WavefrontConfig(grid_shape=(3, 4), batch_size=2, dim=8)
    eng = WavefrontEngine(cfg, nn.ModuleList([nn.Identity() for _ in range(3)]))
    x = torch.randn(2, 4, 8)
    grids = [torch.randn(12, 2, 8) for _ in range(2)]
    ing = fetch_mapped_context(x, grids, 6, eng.routing_map, cfg)
    assert torch.equal(ing[0], grids[0][2]) and torch.equal(ing[1], grids[1][5])
    ing0 = fetch_mapped_context(x, grids, 1, eng.routing_map, cfg)  # row 0 reads x, col 0 zero
    assert torch.equal(ing0[0], x[:, 1, :]) and torch.equal(ing0[1], grids[1][0])
    ing00 = fetch_mapped_context(x, grids, 4, eng.routing_map, cfg)
    assert torch.equal(ing00[1], torch.zeros(2, 8))


# ---------------------------------------------------------------- C ABI
def header_symbols():
    txt = open(os.path.join(REPO, "include", "flb_b200.h")).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(flb_[a-z0-9_]+)\s*\(", txt)))


def test_library_exports_every_header_symbol():
    import flb_native as nat
    syms = header_symbols()
    assert len(syms) >= 12
    for s in syms:
        assert hasattr(nat.lib, s), s
        assert s in nat.PROTOTYPES, f"{s} has no ctypes prototype"


def test_version_and_error_strings():
    import flb_native as nat
    assert "sm_100a" in nat.version()
    st = nat.lib.flb_attn_fwd(None, None, None, None, None, None, None, None, 1, 4, 8, 9, 0, None,
                              0, None)
    assert st == 2  # FLB_ERR_DTYPE, rejected before any device work
    assert "dtype" in nat.lib.flb_last_error().decode()
    with pytest.raises(RuntimeError, match="DTYPE"):
        nat.check(st, "flb_attn_fwd")


def test_attention_argument_validation():
    import flb_native as nat
    L = nat.lib
    nul = [None] * 8
    assert L.flb_attn_fwd(*nul, 1, 4, 300, 0, 0, None, 0, None) == 6  # D > 256 unsupported
    assert L.flb_attn_fwd(*nul, 1, 4, 8, 0, 0, None, 0, None) == 1  # null pointers with work
    # misaligned bf16 pointer
    assert L.flb_attn_fwd(1, 2, 2, 4, 4, 2, 4, None, 1, 4, 8, 2, 0, None, 0, None) == 3
    # empty problems are a no-op
    assert L.flb_attn_fwd(*nul, 0, 4, 8, 0, 0, None, 0, None) == 0
    assert L.flb_attn_bwd_workspace_bytes(8, 16, 64, 2, 1) >= 8 * 16 * 4


def test_index_copy_validation():
    import flb_native as nat
    s = nat.strides(1, 1, 1)
    assert nat.lib.flb_wf_index_copy(None, 0, s, None, None, 0, s, None, -1, 1, 1, 0, None) == 1
    assert nat.lib.flb_wf_index_copy(None, 0, s, None, None, 0, s, None, 0, 1, 1, 0, None) == 0


def test_no_cpu_fallback():
    """CPU tensors are rejected loudly by the product path."""
    from kernels import fused_additive_attention
    q = torch.randn(1, 2, 3, 8)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        fused_additive_attention(q, q, q, torch.randn(2, 1, 8))


def test_backend_module_is_native_and_rejects_cpu():
    import torch.nn as nn
    import wavefront_backend
    from wavefront import WavefrontConfig, WavefrontEngine
    assert wavefront_backend.__file__.endswith(".so")
    cfg = WavefrontConfig(grid_shape=(2, 2), batch_size=1, dim=4)

    class Cell(nn.Module):
        def forward(self, top, left):
            return top + left, top - left

    eng = WavefrontEngine(cfg, nn.ModuleList([Cell(), Cell()]))
    with pytest.raises(Exception, match="CUDA"):
        eng(torch.randn(1, 2, 4))


def test_bench_entry_points_exist():
    """bench.py's arms and modes resolve (the driver runs them only on the GPU box)."""
    import importlib.util
    import os
    import sys
    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "bench.py")
    spec = importlib.util.spec_from_file_location("bench_under_test", path)
    mod = importlib.util.module_from_spec(spec)
    argv = sys.argv
    try:
        sys.argv = ["bench.py"]
        spec.loader.exec_module(mod)
    finally:
        sys.argv = argv
    for name in ("main", "run_flb", "run_reference", "run_ref_engine", "run_profile_case",
                 "a3_sharded", "grid_row_bands", "extra_engine", "extra_flb_e2e",
                 "reference_engine_timing"):
        assert callable(getattr(mod, name, None)), name
    assert mod.profile_traffic("attn_bwd_tc_a2.md") > 1e9
    assert mod.profile_traffic("attn_fwd_tc_a2.md") > 1e9

"""CPU tests: the oracle against independent implementations and the
reference's recorded outputs, the ported routing generators against golden
fixtures produced by the reference's own functions, and the C ABI surface
(loads and validates arguments without a GPU)."""

import ctypes
import json
import re
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import moe_oracle as orc
from src import _lib
from src import routing

GOLDEN = json.loads((Path(__file__).parent / "golden" / "group_sizes.json").read_text())
HEADER = Path(__file__).resolve().parent.parent / "include" / "moe_b200.h"


# ----------------------------------------------------------------------------- golden pins
@pytest.mark.parametrize("case", GOLDEN["benchmark_make_group_sizes"], ids=lambda c: f"M{c['M']}E{c['E']}")
def test_make_group_sizes_matches_reference_function(case):
    got = routing.make_group_sizes(case["M"], case["E"], case["fractions"])
    assert got.tolist() == case["sizes"]


def test_experiment_generators_match_reference_functions():
    for case in GOLDEN["experiment_make_group_sizes"]:
        w = routing.routing_weights(case["E"], case["pattern"])
        assert w.tolist() == case["weights"], case
        got = routing.make_group_sizes_pattern(case["M"], case["E"], case["pattern"])
        assert got.tolist() == case["sizes"], case


def test_group_sizes_recorded_in_reference_results_csv():
    """The 48 routings recorded by the reference's published sweep."""
    assert len(GOLDEN["results_csv_recorded"]) >= 40
    for case in GOLDEN["results_csv_recorded"]:
        got = routing.make_group_sizes_pattern(case["M"], case["E"], case["pattern"])
        assert got.tolist() == case["sizes"], case


def test_reference_generator_errors():
    with pytest.raises(ValueError):
        routing.make_group_sizes(3, 4)
    with pytest.raises(ValueError):
        routing.make_group_sizes(8, 2, [1.0, -1.0])
    with pytest.raises(ValueError):
        routing.routing_weights(4, "nope")


# ----------------------------------------------------------------------------- oracle
def test_gelu_matches_torch_tanh_gelu():
    x = np.linspace(-12, 12, 20001)
    ref = torch.nn.functional.gelu(torch.from_numpy(x), approximate="tanh").numpy()
    assert np.max(np.abs(orc.gelu_tanh(x) - ref)) < 1e-14


def test_ragged_dot_matches_per_group_matmul_and_zero_tail():
    rng = np.random.default_rng(0)
    M, K, N, G = 50, 7, 5, 4
    lhs, rhs = rng.standard_normal((M, K)), rng.standard_normal((G, K, N))
    gs = [10, 0, 25, 9]                      # sum 44 < M
    out = orc.ragged_dot(lhs, rhs, gs)
    offs = np.cumsum([0] + gs)
    for g in range(G):
        a, b = offs[g], offs[g + 1]
        np.testing.assert_allclose(out[a:b], lhs[a:b] @ rhs[g], rtol=1e-13, atol=1e-13)
    assert np.all(out[44:] == 0)


def test_pallas_block_restatement_matches_two_ragged_dots():
    """The restated Pallas control flow (src/kernel.py:9-82): routed rows equal
    ref_ragged_mlp; rows past sum(gs) are never written (fill)."""
    M, D, F, E = 96, 16, 32, 3
    x, wu, wd = routing.make_inputs_numpy(M, D, F, E, seed=1)
    gs = [30, 0, 50]
    y = orc.fused_kernel_blocks(x, wu, wd, gs, BM=16, BF=8, max_group_size=50)
    ref = orc.ref_ragged_mlp(x, wu, wd, gs)
    np.testing.assert_allclose(y[:80], ref[:80], rtol=2e-5, atol=2e-5)
    assert np.all(np.isnan(y[80:]))
    # The reference grid covers cdiv(max_group_size, BM) blocks per expert: a
    # max_group_size below the largest group leaves that group's tail unwritten.
    y2 = orc.fused_kernel_blocks(x, wu, wd, gs, BM=16, BF=8, max_group_size=32)
    assert np.all(np.isfinite(y2[:30])) and np.all(np.isnan(y2[30 + 32:80]))


def test_correctness_metrics_formulas():
    a = np.array([[1.0, -2.0], [3.0, 0.5]])
    b = a + np.array([[0.1, 0.0], [0.0, -0.2]])
    m = orc.correctness_metrics(a, b)
    assert m["max_absolute_error"] == pytest.approx(0.2)
    assert m["l2_relative_error"] == pytest.approx(np.linalg.norm(b - a) / np.linalg.norm(a))
    assert m["normalized_max_error"] == pytest.approx(0.2 / 3.0)


def test_e4m3_decode_matches_torch():
    codes = np.arange(256, dtype=np.uint8)
    ours = orc.e4m3_decode(codes)
    theirs = torch.from_numpy(codes).view(torch.float8_e4m3fn).float().numpy()
    finite = np.isfinite(theirs)
    assert np.array_equal(np.isnan(ours), np.isnan(theirs))
    np.testing.assert_array_equal(ours[finite], theirs[finite])


def test_cpu_reference_port_matches_oracle():
    M, D, F, E = 300, 32, 48, 4
    x, wu, wd = routing.make_inputs_numpy(M, D, F, E, seed=2)
    gs = routing.make_group_sizes(M - 4, E)
    y = orc.time_cpu_reference(x, wu, wd, gs)
    ref = orc.ref_ragged_mlp(x, wu, wd, gs)
    assert orc.correctness_metrics(ref, y)["l2_relative_error"] < 1e-6
    assert np.all(y[M - 4:] == 0)


# ----------------------------------------------------------------------------- routing for the configs
def test_config_routings():
    c3 = routing.zipf_group_sizes(4096, 16, np.random.default_rng(0))
    assert c3.sum() == 4096 and (c3 == 0).sum() >= 3 and c3.max() >= 2048
    c4 = routing.config_group_sizes(routing.CONFIGS["c4"])
    assert c4.sum() == 32768 and len(c4) == 8
    c5 = routing.config_group_sizes(routing.CONFIGS["c5"])
    assert c5.sum() == 65536 and len(c5) == 256
    c1 = routing.config_group_sizes(routing.CONFIGS["c1"])
    assert c1.sum() == 4096


# ----------------------------------------------------------------------------- C ABI
def _declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(moe_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    names = _declared_functions()
    assert {"moe_fused_mlp", "moe_fused_mlp_workspace_size", "moe_last_error"} <= set(names)
    for n in names:
        assert hasattr(L, n), n


def test_abi_validates_arguments_before_any_device_work():
    L = _lib.lib()
    vp = ctypes.c_void_p
    null = vp(0)
    # Negative M -> invalid argument, with a message.
    rc = L.moe_fused_mlp(null, null, null, null, null, null, null, -1, 128, 512, 8, 0, null, 0, null)
    assert rc == -1 and b"bad sizes" in L.moe_last_error()
    # Unknown dtype -> unsupported dtype.
    rc = L.moe_fused_mlp(null, null, null, null, null, null, null, 16, 128, 512, 8, 7, null, 0, null)
    assert rc == -3
    # Unsupported shape (D not a multiple of 256 above 256) -> unsupported shape.
    rc = L.moe_fused_mlp(vp(16), vp(16), vp(16), vp(16), null, null, vp(16), 16, 300, 512, 8, 1, null, 0, null)
    assert rc == -2
    # M == 0 is a no-op.
    assert L.moe_fused_mlp(null, null, null, null, null, null, null, 0, 128, 512, 8, 0, null, 0, null) == 0
    assert L.moe_set_tuning(99, 1) == -1
    assert L.moe_version() >= 100


def test_workspace_sizes():
    L = _lib.lib()
    # f32 small-D: four tf32 weight planes; D=256 adds the two X planes.
    assert L.moe_fused_mlp_workspace_size(65536, 128, 512, 8, 0) == 4 * 8 * 128 * 512 * 4
    assert L.moe_fused_mlp_workspace_size(4096, 256, 2048, 16, 0) == 4 * 16 * 256 * 2048 * 4 + 2 * 4096 * 256 * 4
    # bf16 small-D needs nothing; bf16 large-D holds H (M, F) in bf16.
    assert L.moe_fused_mlp_workspace_size(65536, 128, 512, 8, 1) == 0
    assert L.moe_fused_mlp_workspace_size(32768, 4096, 14336, 8, 1) == 32768 * 14336 * 2


def test_ep_engine_validates_arguments_before_any_device_work():
    L = _lib.lib()
    h = ctypes.c_void_p()
    # rank / world out of range, too many waves, unknown dtype, shape without a kernel.
    assert L.moe_ep_create(2, 2, 4, 1024, 128, 512, 0, 2, 0, ctypes.byref(h)) == -1
    assert L.moe_ep_create(0, 9, 4, 1024, 128, 512, 0, 2, 0, ctypes.byref(h)) == -1
    assert L.moe_ep_create(0, 2, 4, 1024, 128, 512, 0, 9, 0, ctypes.byref(h)) == -1
    assert L.moe_ep_create(0, 2, 1025, 1024, 128, 512, 0, 2, 0, ctypes.byref(h)) == -1
    assert L.moe_ep_create(0, 2, 4, 1024, 128, 512, 7, 2, 0, ctypes.byref(h)) == -3
    assert L.moe_ep_create(0, 2, 4, 1024, 300, 512, 1, 2, 0, ctypes.byref(h)) == -2
    assert h.value is None
    assert L.moe_ep_forward(None, None, None, None, 0, None) == -1
    assert L.moe_ep_launches_per_forward(None) == -1


def test_launch_count_host_side():
    L = _lib.lib()
    assert L.moe_fused_mlp_launch_count(0, 128, 512, 8, 0) == 0
    assert L.moe_fused_mlp_launch_count(-1, 128, 512, 8, 0) == -1
    assert L.moe_fused_mlp_launch_count(16, 128, 512, 8, 9) == -1
    # Two grouped GEMMs for bf16 large D and for e4m3 weights (decoded in
    # shared memory), plus the tf32 split for f32 outside the fused small-D
    # kernels.
    assert L.moe_fused_mlp_launch_count(32768, 4096, 14336, 8, 1) == 2
    assert L.moe_fused_mlp_launch_count(65536, 7168, 2048, 256, 2) == 2
    assert L.moe_fused_mlp_launch_count(16, 384, 512, 8, 1) == 2
    assert L.moe_fused_mlp_launch_count(16, 320, 448, 4, 1) == 2
    assert L.moe_fused_mlp_launch_count(16, 512, 512, 4, 0) == 3
    assert L.moe_fused_mlp_launch_count(16, 320, 448, 4, 2) == 2
    # Rows that do not start on 16-byte boundaries have no kernel (TMA).
    assert L.moe_fused_mlp_launch_count(16, 100, 512, 8, 1) == -2
    assert L.moe_fused_mlp_launch_count(16, 130, 512, 8, 0) == -2
    assert L.moe_fused_mlp_launch_count(16, 320, 440, 8, 2) == -2

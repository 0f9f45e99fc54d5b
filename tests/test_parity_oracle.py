"""GPU: the CUDA path against the CPU oracle on seeded inputs, every mode.

fp32 cases at rel-L2 <= 1e-5, bf16 cases (bf16 inputs, fp32 state) at <= 2e-2, on
y, S_end, Z_end, the new omega buffer and every input gradient.
"""
import pytest
import torch

from atlas_rnn_b200 import memory_recurrence
from atlas_rnn_b200.workloads import CONFIGS, Workload, make_inputs, shrink
from tests.helpers import TOL_BF16, TOL_F32, oracle_run, rel_l2

pytestmark = pytest.mark.gpu


def run_case(w: Workload, seed=0, state_scale=0.1, tol=None, separate_sref=False, chunk=0, mutate=None):
    tol = tol if tol is not None else (TOL_F32 if w.dtype == torch.float32 else TOL_BF16)
    inp = make_inputs(w, seed=seed, device="cuda", state_scale=state_scale)
    if mutate is not None:
        mutate(inp)
    g = torch.Generator().manual_seed(seed + 7)
    S_ref = (0.1 * torch.randn(w.N, w.d_v, w.d_phi, generator=g)).cuda() if separate_sref else None
    leaves = {n: (t.clone().requires_grad_(True) if t is not None else None) for n, t in inp.items()
              if n not in ("dy", "proj")}
    if S_ref is not None:
        S_ref = S_ref.clone().requires_grad_(True)
    gm = "window" if w.gate == "window" else "token"
    y, S_end, Z_end, nb = memory_recurrence(
        leaves["k"], leaves["q"], leaves["v"], leaves["lr"], leaves["decay"], leaves["beta"], leaves["gate"],
        S_ref=S_ref if S_ref is not None else leaves["S0"], S0=leaves["S0"], Z0=leaves["Z0"],
        omega_buffer=leaves["omega_buffer"], window=w.window, gate_mode=gm, fmap_mode=w.fmap_mode,
        fmap_degree=w.fmap_degree, proj=inp["proj"], chunk=chunk)
    gen = torch.Generator().manual_seed(seed + 11)
    up = {"y": inp["dy"].float().cpu(),
          "S_end": torch.randn(S_end.shape, generator=gen),
          "Z_end": torch.randn(S_end.shape, generator=gen) if Z_end is not None else None,
          "buf_out": torch.randn(nb.shape, generator=gen) if nb is not None else None}
    ref_in = dict(inp)
    out_ref, g_ref = oracle_run(ref_in, w.window, gm if w.gate != "none" else None, w.fmap_mode, w.fmap_degree,
                                up=up, S_ref=S_ref)
    mine = {"y": y, "S_end": S_end, "Z_end": Z_end, "buf_out": nb}
    errs = {}
    for n, o in mine.items():
        if o is not None:
            errs[n] = rel_l2(o.float(), out_ref[n])
    pairs = [(mine[n], up[n].to(mine[n].dtype).cuda()) for n in mine if mine[n] is not None]
    torch.autograd.backward([p[0] for p in pairs], [p[1] for p in pairs])
    for n, t in leaves.items():
        if t is not None and n in g_ref:
            errs["d_" + n] = rel_l2(t.grad.float(), g_ref[n])
    if S_ref is not None:
        errs["d_S_ref"] = rel_l2(S_ref.grad, g_ref["S_ref"])
    bad = {k: v for k, v in errs.items() if not v < tol}
    assert not bad, (bad, errs)
    return errs


def W(name, T, d=32, dv=None, e=1, gate="none", fm="off", deg=1, mom=True, dtype=torch.float32, N=(1, 3),
      dphi=None):
    dv = dv or d
    return Workload(name, N[0], N[1], T, d, dphi or d, dv, e, gate, fm, deg, mom, dtype, 0)


CASES_F32 = [
    W("titans", 100),
    W("titans_nomom", 77, mom=False),
    W("omega_e2_token", 65, e=2, gate="token"),
    W("omega_e4_window", 70, e=4, gate="window"),
    W("omega_e4_elem3", 64, e=4, gate="token", fm="elementwise", deg=3),
    W("omega_e16_token", 97, e=16, gate="token", d=64),
    W("omega_e5_nogate", 33, e=5),
    W("rect_dv48_dphi32", 50, d=32, dv=48, e=3, gate="token"),
    W("tensor_fmap", 40, d=8, dphi=24, e=3, gate="token", fm="tensor", deg=2),
    W("t1", 1, e=3, gate="token"),
    W("t_lt_window", 3, e=8, gate="window"),
    W("t_eq_chunk", 32, e=2, gate="token"),
    W("t_chunk_plus1", 33, e=2, gate="token"),
    W("t_chunk_minus1", 31, e=4, gate="window"),
    W("d128", 70, d=128, e=4, gate="window", fm="elementwise", deg=2),
]


@pytest.mark.parametrize("w", CASES_F32, ids=lambda w: w.name)
def test_fp32_vs_oracle(native_lib, w):
    run_case(w)


@pytest.mark.parametrize("w", CASES_F32[:6], ids=lambda w: w.name)
def test_fp32_separate_sref(native_lib, w):
    run_case(w, separate_sref=True)


@pytest.mark.parametrize("w", [W("bf16_titans", 130, d=64, dtype=torch.bfloat16),
                               W("bf16_omega_window", 99, d=64, e=4, gate="window", fm="elementwise", deg=2,
                                 dtype=torch.bfloat16)], ids=lambda w: w.name)
@pytest.mark.parametrize("pad", ["1", "0"], ids=["padded_tc", "cuda_cores"])
def test_bf16_vs_oracle(native_lib, monkeypatch, w, pad):
    """bf16 heads under 128 run the tensor-core kernels zero-padded (default) or the
    CUDA-core kernels (ATLAS_MEM_PAD128=0)."""
    monkeypatch.setenv("ATLAS_MEM_PAD128", pad)
    run_case(w)


# bf16 heads narrower than 128 on the zero-padded tensor-core path
CASES_PAD = [
    W("pad_c3_like_e8_token_elem", 300, d=64, e=8, gate="token", fm="elementwise", deg=2, dtype=torch.bfloat16,
      N=(2, 3)),
    W("pad_titans_d32_nomom", 140, d=32, mom=False, dtype=torch.bfloat16),
    W("pad_rect_dv48_dphi32", 133, d=32, dv=48, e=3, gate="token", dtype=torch.bfloat16),
    W("pad_e16_window_d64", 200, d=64, e=16, gate="window", dtype=torch.bfloat16),
    W("pad_short_t3", 3, d=64, e=4, gate="token", dtype=torch.bfloat16),
]


@pytest.mark.parametrize("w", CASES_PAD, ids=lambda w: w.name)
def test_bf16_padded_tensor_core_path(native_lib, w):
    run_case(w, state_scale=0.1)


def test_config0_full(native_lib):
    """Benchmark config 0 at full size (fp32)."""
    run_case(CONFIGS[0], state_scale=0.0)
    run_case(CONFIGS[0], state_scale=0.1, seed=1)


def test_config1_slice(native_lib):
    """Benchmark config 1 (bf16, e=4, window gates, elementwise g=2) on a batch*head slice,
    from a zero state (the benchmark's) and from a non-zero S0 / Z0 / omega buffer
    (scale 0.1, as the reference's tests use: test_rnn_all.py:469-470,551-553)."""
    run_case(shrink(CONFIGS[1], B=1, H=2, T=1024), state_scale=0.0)
    run_case(shrink(CONFIGS[1], B=1, H=2, T=4096), state_scale=0.1, seed=4)


# ---- the clamp of S_end (rnn_memory.py:372-373,701-702) driven into saturation -------------
def _saturate(inp):
    """alpha close to 1 and |S0| of order 150, so a large share of S_T lies beyond +-100:
    S_end is clamped there and its gradient is zero (torch.clamp's rule)."""
    g = torch.Generator().manual_seed(99)
    dec = inp["decay"]
    inp["decay"] = (0.999 + 0.001 * torch.rand(dec.shape, generator=g)).to(dec.dtype).to(dec.device)
    inp["S0"] = (1500.0 * inp["S0"]).contiguous()  # S0 was 0.1 N(0,1)
    S_T_est = inp["S0"]
    assert (S_T_est.abs() > 100).float().mean() > 0.3


CASES_CLAMP = [
    W("clamp_f32_e4_token", 90, e=4, gate="token"),
    W("clamp_f32_nomom", 70, mom=False),
    W("clamp_tc_e4_window_elem", 260, d=128, e=4, gate="window", fm="elementwise", deg=2, dtype=torch.bfloat16),
    W("clamp_tc_nomom", 200, d=128, mom=False, dtype=torch.bfloat16),
    W("clamp_padded_d64_e8", 150, d=64, e=8, gate="token", dtype=torch.bfloat16),
]


@pytest.mark.parametrize("w", CASES_CLAMP, ids=lambda w: w.name)
def test_clamp_saturated(native_lib, w):
    """S_end, Z_end and every input gradient against the oracle with the clamp active
    (CUDA-core fp32 path, tensor-core bf16 path, padded tensor-core path). S_ref is a
    separate state of the usual scale (0.1), so the deltas stay of order one and the
    bf16 tolerance measures the clamp, not bf16 rounding of deltas of order 100."""
    run_case(w, state_scale=0.1, mutate=_saturate, separate_sref=True)


def test_config4_slice(native_lib):
    """Benchmark config 4 (tensor feature map 64 -> 256, e=16) on a small slice."""
    run_case(shrink(CONFIGS[4], B=1, H=1, T=160), state_scale=0.1)


@pytest.mark.parametrize("chunk", [16, 24, 64])
def test_chunk_invariance(native_lib, chunk):
    """The internal chunk is only a tiling (reference: test_rnn_all.py:335-374)."""
    run_case(W("chunk_inv", 90, e=4, gate="token"), chunk=chunk)


# bf16, head size 128: the tensor-core kernels run for these (ATLAS_MEM_TC selects them)
CASES_TC = [
    W("tc_titans", 300, d=128, dtype=torch.bfloat16),
    W("tc_omega_e4_window_elem", 257, d=128, e=4, gate="window", fm="elementwise", deg=2, dtype=torch.bfloat16),
    W("tc_omega_e16_token", 200, d=128, e=16, gate="token", dtype=torch.bfloat16),
    W("tc_nomom_e2", 130, d=128, e=2, gate="token", mom=False, dtype=torch.bfloat16),
    W("tc_short", 5, d=128, e=3, gate="token", dtype=torch.bfloat16),
    W("tc_tensor_fmap", 150, d=8, dphi=128, dv=128, e=3, gate="token", fm="tensor", deg=2, dtype=torch.bfloat16),
]


@pytest.mark.parametrize("w", CASES_TC, ids=lambda w: w.name)
@pytest.mark.parametrize("state_scale", [0.0, 0.1])
def test_bf16_tensor_core_path(native_lib, w, state_scale):
    run_case(w, state_scale=state_scale)


# tensor feature map on tensor cores (bf16, d_k in {16, 32, 64}, d_phi up to 256): the
# [x; vec(x x^T)] Proj GEMM of rnn_memory.py:125-130 and its backward
CASES_FMAP_TC = [
    W("fmap_tc_d16_phi128_tcrec", 300, d=16, dphi=128, dv=128, e=3, gate="token", fm="tensor", deg=2,
      dtype=torch.bfloat16),
    W("fmap_tc_d32_phi64", 200, d=32, dphi=64, dv=48, e=2, gate="window", fm="tensor", deg=2, dtype=torch.bfloat16),
    W("fmap_tc_d64_phi256_e16", 260, d=64, dphi=256, dv=128, e=16, gate="token", fm="tensor", deg=2,
      dtype=torch.bfloat16),
    # d_phi = 256 with a narrower value head: the column parts run the zero-padded tensor-core path
    W("fmap_tc_d32_phi256_dv64_window", 200, d=32, dphi=256, dv=64, e=4, gate="window", fm="tensor", deg=2,
      dtype=torch.bfloat16),
]


@pytest.mark.parametrize("w", CASES_FMAP_TC, ids=lambda w: w.name)
def test_tensor_fmap_tensor_cores(native_lib, w):
    run_case(w, state_scale=0.1)

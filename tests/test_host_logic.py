"""CPU: host-side decisions and helpers around the kernels (no kernel launches):
the LM's sampling helpers (rnn_transformer.py:42-59), which heads take the zero-padded
tensor-core route, and which cells prepare their heads in one pass."""
import torch

import atlas_rnn_b200 as A
from atlas_rnn_b200 import _lib
from atlas_rnn_b200.headprep import HEAD_DIMS
from atlas_rnn_b200.ops import Spec, _pad_to_tc
from atlas_rnn_b200.rnn_transformer import gumbel_sample, min_p_filter


def test_min_p_filter_keeps_tokens_above_the_fraction_of_the_top():
    logits = torch.log(torch.tensor([[0.5, 0.3, 0.04, 0.16]]))
    out = min_p_filter(logits, min_p=0.1)  # limit = 0.05: only 0.04 goes
    assert torch.isinf(out[0, 2]) and out[0, 2] < 0
    assert torch.equal(out[0, [0, 1, 3]], logits[0, [0, 1, 3]])


def test_gumbel_sample_at_zero_temperature_is_argmax():
    t = torch.tensor([[0.1, 2.0, -1.0], [3.0, 0.0, 0.5]])
    assert torch.equal(gumbel_sample(t, temperature=0.0), torch.tensor([[1], [0]]))


def test_padded_tensor_core_route(monkeypatch):
    bf, f32 = torch.bfloat16, torch.float32
    off = Spec(window=8, gate_mode=_lib.GATE_TOKEN, fmap_mode="elementwise", fmap_degree=2, momentum=True)
    assert _pad_to_tc(off, bf, 64, 64, 64)
    assert not _pad_to_tc(off, f32, 64, 64, 64)          # fp32 operands stay on the CUDA cores
    assert not _pad_to_tc(off, bf, 128, 128, 128)        # already the kernels' size
    assert not _pad_to_tc(off, bf, 64, 64, 256)          # d_v above 128
    tensor = Spec(window=3, gate_mode=_lib.GATE_TOKEN, fmap_mode="tensor", fmap_degree=2, momentum=True)
    assert not _pad_to_tc(tensor, bf, 8, 64, 64)         # tensor map: d_phi != d_k
    wide = Spec(window=17, gate_mode=_lib.GATE_TOKEN, fmap_mode="off", fmap_degree=1, momentum=True)
    assert not _pad_to_tc(wide, bf, 64, 64, 64)          # window above 16
    monkeypatch.setenv("ATLAS_MEM_PAD128", "0")
    assert not _pad_to_tc(off, bf, 64, 64, 64)


def test_head_prep_route_needs_bf16_and_a_supported_head():
    cell = A.OmegaRNNMemoryCell(dim=128, dim_head=64, heads=2, omega_window=8, use_omega_gate=True)
    x = torch.zeros(1, 4, 128)
    assert not cell._head_prep_ok(x, 4)                  # CPU tensors never take it
    assert HEAD_DIMS == (32, 64, 96, 128)                # one warp per row, d / 32 elements a lane


def test_lm_parameter_count_of_the_benchmark_config():
    """Config 3's LM: about 86 M parameters (12 layers, d_model 768, SwiGLU 2048)."""
    m = A.RNNMemoryTransformer(num_tokens=256, dim=768, depth=12, block_type="lmm", heads=12, dim_head=64,
                               omega_window=8, use_omega_gate=True, poly_mode="elementwise", poly_degree=2)
    n = sum(p.numel() for p in m.parameters())
    assert 85e6 < n < 87e6
    assert m.layers[0].ff[1].out_features == 2 * 2048

"""The LMM language model (RNNMemoryTransformer, block_type 'lmm') as a drop-in for the
reference's rnn_transformer.py: the reference state_dict loads unchanged (CPU), and on the
GPU the next-token loss, logits, every parameter gradient and the logits of one-token
cached steps match the reference's golden vectors (fp32 vs the reference in fp64)."""
import pytest
import torch

from tests.helpers import TOL_F32, golden_files, load, rel_l2

LM_TOL_GRAD = 1e-4  # parameter gradients summed over all tokens through two blocks, fp32


def build(name):
    import atlas_rnn_b200 as A
    from tests.golden.make_golden import LM_CASES
    kw, B, T, steps = LM_CASES[name]
    z = load(golden_files(name)[0])
    m = A.RNNMemoryTransformer(**kw)
    m.load_state_dict({k[3:]: torch.from_numpy(v).float() for k, v in z.items() if k.startswith("sd.")})
    return m, z


@pytest.mark.parametrize("path", golden_files("lm_"), ids=lambda p: p.split("/")[-1])
def test_reference_state_dict_loads(path):
    name = path.split("/")[-1][:-4]
    m, z = build(name)
    ours = dict(m.named_parameters())
    assert sorted(ours) == sorted(k[5:] for k in z if k.startswith("grad."))


def test_attention_block_types_are_refused():
    import atlas_rnn_b200 as A
    for bt in ("mag", "mal", "mac"):
        with pytest.raises(ValueError):
            A.RNNMemoryTransformer(num_tokens=16, dim=8, depth=1, block_type=bt, heads=1, dim_head=8)


@pytest.mark.gpu
@pytest.mark.parametrize("path", golden_files("lm_"), ids=lambda p: p.split("/")[-1])
def test_lm_matches_reference_golden(native_lib, path):
    name = path.split("/")[-1][:-4]
    m, z = build(name)
    m = m.cuda()
    tokens = torch.from_numpy(z["tokens"]).cuda()
    loss, logits, _, _ = m(tokens, return_loss=True, return_cache=True)
    assert abs(loss.item() - float(z["loss"])) / abs(float(z["loss"])) < TOL_F32
    assert rel_l2(logits, z["logits"]) < TOL_F32
    loss.backward()
    worst = max((rel_l2(p.grad, z["grad." + n]), n) for n, p in m.named_parameters())
    assert worst[0] < LM_TOL_GRAD, worst
    st = None
    with torch.no_grad():
        for s in range(z["step_tokens"].shape[0]):
            lg, st, _ = m(torch.from_numpy(z["step_tokens"][s]).cuda(), mem_states=st, return_cache=True)
            assert rel_l2(lg, z["step_logits"][s]) < TOL_F32, (s, rel_l2(lg, z["step_logits"][s]))


@pytest.mark.gpu
def test_generate_shape_and_training_step(native_lib):
    """rnn_all transformer tests' shape of generate and a few optimiser steps with finite loss."""
    import math
    import atlas_rnn_b200 as A
    torch.manual_seed(0)
    m = A.LongTermMemoryModel(num_tokens=256, dim=64, depth=1, heads=2, dim_head=16, omega_window=4,
                              use_omega_gate=True, poly_mode="elementwise", poly_degree=2).cuda()
    out = m.generate(torch.randint(0, 256, (1, 4), device="cuda"), max_length=12)
    assert out.shape == (1, 12)
    m.train()
    opt = torch.optim.Adam(m.parameters(), lr=1e-4)
    for _ in range(3):
        loss = m(torch.randint(0, 256, (2, 16), device="cuda"), return_loss=True)
        opt.zero_grad()
        loss.backward()
        opt.step()
        assert math.isfinite(loss.item())

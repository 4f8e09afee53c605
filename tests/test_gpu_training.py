"""The config-4 training step on the GPU (training.py): the model's forward on
the B200 ops equals the same parameters through the CPU oracle, and a few
optimisation steps under bf16 autocast run the tensor-core mixer kernels and
lower the loss on a fixed batch."""
import copy

import pytest
import torch

from conftest import load_pkg
from test_training import _training, cpu_mixer_cls

pytestmark = pytest.mark.gpu


def test_model_forward_and_gradient_match_cpu_oracle():
    tr = _training()
    torch.manual_seed(5)
    cpu = tr.LanguageModel(211, 128, 2, 2, "delta", chunk=64, mixer_cls=cpu_mixer_cls())
    gpu = tr.LanguageModel(211, 128, 2, 2, "delta", chunk=64)
    gpu.load_state_dict(cpu.state_dict())
    gpu = gpu.cuda()
    g = torch.Generator().manual_seed(6)
    idx = torch.randint(0, 211, (2, 129), generator=g)
    _, lc = cpu(idx[:, :-1], idx[:, 1:])
    lc.backward()
    _, lg = gpu(idx[:, :-1].cuda(), idx[:, 1:].cuda())   # fp32: the exact-fp32 kernels
    lg.backward()
    assert abs(lg.item() - lc.item()) <= 1e-5 * abs(lc.item())
    for (n, pc), pg in zip(cpu.named_parameters(), gpu.parameters()):
        e = (pg.grad.cpu() - pc.grad).abs().max().item() / (pc.grad.abs().max().item() + 1e-12)
        assert e < 1e-3, n


@pytest.fixture
def tf32_matmul():
    """TF32 GEMMs as the reference's trainer enables them, restored afterwards
    (other tests compare fp32 GEMMs against the CPU)."""
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


@pytest.mark.parametrize("inner", ["delta", "muon", "adam"])
def test_training_steps_lower_the_loss(inner, tf32_matmul):
    pkg = load_pkg()
    tr = _training()
    torch.manual_seed(7)
    model = tr.LanguageModel(1000, 256, 2, 4, inner, chunk=64).cuda()   # dh 64
    opts = tr.build_optimizers(model, muon_lr=0.02, adam_lr=3e-3)
    g = torch.Generator().manual_seed(8)
    idx = torch.randint(0, 1000, (4, 257), generator=g).cuda()
    L = pkg._lib
    L.prof_report()
    L.prof_enable(True)
    losses = [tr.train_step(model, opts, idx[:, :-1], idx[:, 1:]).item() for _ in range(6)]
    torch.cuda.synchronize()
    L.prof_enable(False)
    names = set(L.prof_report())
    fwd = "chunk_fwd_muon_tc" if inner == "muon" else "chunk_fwd_tc"
    assert {fwd, "mixer_prologue_fwd", "head_rmsnorm_bwd"} <= names, names
    assert names & {"chunk_bwd2_tc", "chunk_bwd_fused_tc"}, names   # token gradients
    assert all(l == l for l in losses)            # finite
    assert losses[-1] < losses[0] - 0.05, losses


def test_b200_model_matches_reference_lm_logits():
    """The reference trainer's own LM (weights and logits recorded in
    tests/golden/lm.pt, d_model 64, 2 heads of 32, chunk 32) loaded into this
    package's LanguageModel on the GPU: the mixer runs the B200 prologue,
    chunk and epilogue ops (fp32, head dim 32: the exact chunk kernels) and gives
    the reference's logits."""
    import os
    from conftest import ROOT
    tr = _training()
    gold = torch.load(os.path.join(ROOT, "tests", "golden", "lm.pt"), weights_only=False)
    for inner, g in gold.items():
        m = tr.LanguageModel(61, 64, 2, 2, inner, chunk=32, ns_steps=3)
        m.load_state_dict(g["state"])
        m = m.cuda()
        with torch.no_grad():
            logits, loss = m(g["idx"][:, :-1].cuda(), g["idx"][:, 1:].cuda())
        err = (logits.cpu() - g["logits"]).abs().max().item() / g["logits"].abs().max().item()
        assert err < 1e-4, (inner, err)
        assert abs(loss.item() - g["loss"].item()) < 1e-4 * abs(g["loss"].item()), inner
        gm = m.gate_means()
        for k in ("alpha", "beta", "mu"):
            assert abs(gm[k] - g["gate_means"][k]) < 1e-5, (inner, k)

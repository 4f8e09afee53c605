"""The config-4 training step's host logic on CPU (training.py): the batched
msign against the reference's formula, the outer Muon update, the optimiser
split, and data parallelism with two gloo ranks (DDP's all-reduced gradient
and one full step equal the single-process run on the whole batch).  The
mixer's B200 ops need a GPU, so the CPU model runs the same mixer parameters
through the oracle mixer core."""
import os
import socket

import torch
import torch.multiprocessing as mp
import torch.nn.functional as F

from conftest import ROOT, load_pkg


def _training():
    import importlib
    load_pkg()
    from conftest import PKG_NAME
    return importlib.import_module(PKG_NAME + ".training")


def ref_msign(M, steps=5, eps=1e-7):
    """train_ablation.py:60-73 restated (one matrix)."""
    X = M.float()
    tall = X.shape[-2] > X.shape[-1]
    if tall:
        X = X.mT
    X = X / (X.norm(dim=(-2, -1), keepdim=True) + eps)
    a, b, c = 3.4445, -4.7750, 2.0315
    for _ in range(steps):
        A = X @ X.mT
        X = a * X + (b * A + c * (A @ A)) @ X
    return X.mT if tall else X


def test_batched_msign_matches_reference_formula():
    tr = _training()
    g = torch.Generator().manual_seed(0)
    for shape in ((3, 40, 24), (2, 24, 40), (4, 32, 32), (36, 64)):
        M = torch.randn(*shape, generator=g)
        want = ref_msign(M) if M.dim() == 2 else torch.stack([ref_msign(m) for m in M])
        assert (tr.msign(M) - want).abs().max().item() < 5e-6, shape


def test_outer_muon_step_matches_reference_update():
    tr = _training()
    g = torch.Generator().manual_seed(1)
    ps = [torch.nn.Parameter(torch.randn(48, 16, generator=g)) for _ in range(2)]
    ps.append(torch.nn.Parameter(torch.randn(16, 48, generator=g)))
    before = [p.detach().clone() for p in ps]
    grads = [torch.randn(p.shape, generator=g) for p in ps]
    opt = tr.OuterMuon(ps, lr=0.02, momentum=0.95, weight_decay=0.1)
    for p, gr in zip(ps, grads):
        p.grad = gr.clone()
    opt.step()
    for p, p0, gr in zip(ps, before, grads):
        buf = gr                             # zero buffer, then buf = 0.95 * 0 + g
        u = ref_msign(gr + 0.95 * buf)        # Nesterov
        scale = max(1.0, p.shape[0] / p.shape[1]) ** 0.5
        want = p0 * (1 - 0.02 * 0.1) - 0.02 * scale * u
        assert (p.detach() - want).abs().max().item() < 1e-5


def test_optimizer_split():
    tr = _training()
    m = tr.LanguageModel(100, 64, 2, 2, "delta")
    muon, adamw = tr.build_optimizers(m)
    hidden = {id(p) for g in muon.param_groups for p in g["params"]}
    other = {id(p) for g in adamw.param_groups for p in g["params"]}
    assert id(m.emb.weight) in other and id(m.emb.weight) not in hidden   # tied head too
    for blk in m.blocks:
        mx = blk.mixer
        for p in (mx.qkv.weight, mx.gates.weight, mx.out.weight, blk.mlp[0].weight, blk.mlp[2].weight):
            assert id(p) in hidden
        for p in (mx.conv.weight, mx.conv.bias, mx.gates.bias, mx.norm.weight, blk.n1.weight):
            assert id(p) in other
    assert len(hidden & other) == 0
    assert len(hidden) + len(other) == len(list(m.parameters()))
    bias = m.blocks[0].mixer.gates.bias.view(3, 2)
    assert torch.equal(bias[:, 0], torch.tensor([3.0, -1.0, 1.0]))


def cpu_mixer_cls():
    """MixerLayer with its forward on the CPU oracle (same parameters)."""
    tr = _training()
    import oracle

    class CpuMixer(tr.MixerLayer):
        def forward(self, x):
            B, T, D = x.shape
            H, dh = self.h, self.dh
            qkv = self.conv(self.qkv(x).transpose(1, 2))[..., :T].transpose(1, 2)
            q, k, v = F.silu(qkv).chunk(3, dim=-1)
            q = F.normalize(q.reshape(B, T, H, dh).transpose(1, 2), dim=-1)
            k = F.normalize(k.reshape(B, T, H, dh).transpose(1, 2), dim=-1)
            v = v.reshape(B, T, H, dh).transpose(1, 2)
            g = torch.sigmoid(self.gates(x)).view(B, T, self.n_gates, H).permute(2, 0, 3, 1)
            nu = g[3] if self.n_gates == 4 else None
            rule = {"delta": 0, "muon": 1, "adam": 2}[self.inner]
            o = oracle.mixer_core_forward(q, k, v, g[0], g[1], g[2], nu, rule, self.ns_steps,
                                          self.chunk)
            return self.out(self.norm(o).transpose(1, 2).reshape(B, T, D))

    return CpuMixer


def _model(seed):
    tr = _training()
    torch.manual_seed(seed)
    return tr.LanguageModel(97, 32, 2, 2, "delta", chunk=16, mixer_cls=cpu_mixer_cls())


def _batch():
    g = torch.Generator().manual_seed(3)
    idx = torch.randint(0, 97, (4, 32), generator=g)
    return idx[:, :-1].contiguous()[:, :16], idx[:, 1:17].contiguous()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ddp_worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    tr = _training()
    model = torch.nn.parallel.DistributedDataParallel(_model(0))
    idx, tgt = _batch()
    lo, hi = rank * 2, rank * 2 + 2
    _, loss = model(idx[lo:hi], tgt[lo:hi])
    loss.backward()
    grads = {n: p.grad.clone() for n, p in model.module.named_parameters()}
    opts = tr.build_optimizers(model)
    torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    for o in opts:
        o.step()
    if rank == 0:
        torch.save({"grads": grads, "params": dict(model.module.state_dict())},
                   os.path.join(out_dir, "ddp.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_ddp_step_equals_single_process(tmp_path):
    """DDP averages the two ranks' gradients over NCCL's CPU twin (gloo); with
    equal shards that is the gradient of the mean loss on the whole batch, and
    the step that follows (clipping, Muon, AdamW) equals the single-process
    step on it."""
    world = 2
    mp.start_processes(_ddp_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    tr = _training()
    model = _model(0)
    idx, tgt = _batch()
    _, loss = model(idx, tgt)
    loss.backward()
    got = torch.load(tmp_path / "ddp.pt")
    for n, p in model.named_parameters():
        e = (got["grads"][n] - p.grad).abs().max().item()
        assert e <= 1e-5 * (p.grad.abs().max().item() + 1e-12) + 1e-7, n
    opts = tr.build_optimizers(model)
    torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    for o in opts:
        o.step()
    for n, t in model.state_dict().items():
        assert (got["params"][n] - t).abs().max().item() < 1e-5, n


def test_lr_schedule_matches_reference_factor():
    """lr_factor restates train_ablation.py:310-314; LrSchedule scales the
    groups' rates from their values at construction."""
    import math
    tr = _training()
    assert tr.lr_factor(0, 500, 9600) == 1 / 500
    assert tr.lr_factor(499, 500, 9600) == 1.0
    assert abs(tr.lr_factor(500 + 9100 // 2, 500, 9600) - (0.1 + 0.45)) < 1e-12
    assert abs(tr.lr_factor(20000, 500, 9600) - 0.1) < 1e-12
    m = tr.LanguageModel(50, 32, 1, 2, "delta")
    opts = tr.build_optimizers(m, muon_lr=0.02, adam_lr=4e-4)
    sched = tr.LrSchedule(opts, warmup=10, total=100)
    for step in (0, 4, 9, 55, 99):
        fac = sched.set_step(step)
        assert math.isclose(opts[0].param_groups[0]["lr"], 0.02 * fac)
        assert math.isclose(opts[1].param_groups[0]["lr"], 4e-4 * fac)


def _lm_golden():
    return torch.load(os.path.join(ROOT, "tests", "golden", "lm.pt"), weights_only=False)


def test_model_matches_reference_lm_weights_and_logits():
    """The fixture holds the reference trainer's own LM (train_ablation.py:
    197-246) per inner rule: its seeded initialisation, and its logits on a
    token batch.  The same seed gives this package's LanguageModel the same
    weights under the same names, and with the mixer core on the oracle the
    same logits."""
    tr = _training()
    gold = _lm_golden()
    for inner, g in gold.items():
        torch.manual_seed(0)
        m = tr.LanguageModel(61, 64, 2, 2, inner, chunk=32, ns_steps=3, mixer_cls=cpu_mixer_cls())
        sd = m.state_dict()
        assert set(sd) == set(g["state"]), inner
        for k, v in g["state"].items():
            assert torch.equal(sd[k], v), (inner, k)
        with torch.no_grad():
            logits, loss = m(g["idx"][:, :-1], g["idx"][:, 1:])
        err = (logits - g["logits"]).abs().max().item() / g["logits"].abs().max().item()
        assert err < 1e-4, (inner, err)
        assert abs(loss.item() - g["loss"].item()) < 1e-5 * abs(g["loss"].item()), inner


def test_run_log_and_checkpoint_formats(tmp_path):
    """RunLog writes the reference's CSV header and row formats and its
    crash-safe {meta, log} JSON (train_ablation.py:426-444, 497-519);
    save_checkpoint writes its checkpoint dictionary (:516-528), which
    load_checkpoint turns back into the same model, and a checkpoint holding
    the reference LM's own state dict loads the same way."""
    import json
    tr = _training()
    m = _model(4)
    opts = tr.build_optimizers(m)
    sched = tr.LrSchedule(opts, warmup=2, total=4)
    idx, tgt = _batch()
    log = tr.RunLog(str(tmp_path), "outer-muon_inner-delta", dict(condition="outer-muon_inner-delta"))
    for step in range(1, 4):
        sched.set_step(step - 1)
        for o in opts:
            o.zero_grad(set_to_none=True)
        _, loss = m(idx, tgt)
        loss.backward()
        gn = torch.nn.utils.clip_grad_norm_(m.parameters(), 1.0).item()
        for o in opts:
            o.step()
        vl, vp = tr.evaluate(m, [(idx, tgt)], amp=False)
        log.row(step, loss.item(), vl, vp, opts[0].param_groups[0]["lr"], gn, 123.4,
                dict(alpha=0.9, beta=0.3, mu=0.7), 1.5 * step, tokens_seen=step * idx.numel())
    log.finish(dict(final_val_loss=vl, final_val_ppl=vp))
    lines = open(tmp_path / "outer-muon_inner-delta.csv").read().splitlines()
    assert lines[0] == ("step,train_loss,val_loss,val_ppl,lr_hidden,grad_norm,tok_s,"
                        "alpha,beta,mu,nu,elapsed_s")
    assert len(lines) == 4
    cells = lines[3].split(",")
    assert cells[0] == "3" and cells[-1] == "4.5" and cells[-2] == "nan" and cells[6] == "123.4"
    assert len(cells[1].split(".")[1]) == 6 and "e" in cells[4]
    meta = json.load(open(tmp_path / "outer-muon_inner-delta_metrics.json"))
    assert set(meta) == {"meta", "log"} and len(meta["log"]) == 3
    assert meta["meta"]["final"]["final_val_loss"] == vl
    assert meta["log"][2]["tokens_seen"] == 3 * idx.numel()
    assert not os.path.exists(tmp_path / "outer-muon_inner-delta_metrics.json.tmp")
    ck = tmp_path / "c.pt"
    tr.save_checkpoint(str(ck), m, vocab=97, d_model=32, n_layers=2, n_heads=2, inner="delta",
                       chunk=16, outer="muon", step=3, seed=0, data_seed=1, args={"lr": 1},
                       final_val_loss=vl, final_val_ppl=vp)
    m2, d = tr.load_checkpoint(str(ck), mixer_cls=cpu_mixer_cls())
    assert d["condition"] == "outer-muon_inner-delta" and d["step"] == 3
    assert set(d) >= {"model_state", "model_config", "outer", "inner", "seed", "data_seed",
                      "args", "torch_version", "final_val_loss", "final_val_ppl"}
    for k, v in m.state_dict().items():
        assert torch.equal(m2.state_dict()[k], v), k
    g = _lm_golden()["muon"]
    ref_ck = tmp_path / "ref.pt"
    torch.save(dict(model_state=g["state"], model_config=dict(
        vocab=61, d_model=64, n_layers=2, n_heads=2, inner="muon", chunk=32)), ref_ck)
    m3, _ = tr.load_checkpoint(str(ref_ck), mixer_cls=cpu_mixer_cls())
    with torch.no_grad():
        logits, _ = m3(g["idx"][:, :-1])
    assert (logits - g["logits"]).abs().max().item() < 1e-4 * g["logits"].abs().max().item()


def test_outer_adam_condition():
    """outer 'adam' puts the hidden matrices on AdamW too
    (train_ablation.py:303-307)."""
    tr = _training()
    m = tr.LanguageModel(50, 32, 1, 2, "delta")
    opts = tr.build_optimizers(m, outer="adam")
    assert all(isinstance(o, torch.optim.AdamW) for o in opts)
    assert opts[0].param_groups[0]["betas"] == (0.9, 0.95)


def test_swiglu_variant():
    """The SwiGLU MLP (the config-4 benchmark description's variant): all
    three of its matrices are hidden matrices for Muon, the residual output
    projection gets the scaled init, and a step runs."""
    import math
    tr = _training()
    torch.manual_seed(2)
    m = tr.LanguageModel(97, 32, 2, 2, "delta", chunk=16, mixer_cls=cpu_mixer_cls(), mlp="swiglu")
    muon, _ = tr.build_optimizers(m)
    hidden = {id(p) for g in muon.param_groups for p in g["params"]}
    for blk in m.blocks:
        for lin in (blk.mlp.gate, blk.mlp.up, blk.mlp.out):
            assert id(lin.weight) in hidden
        assert blk.mlp[2] is blk.mlp.out
        assert blk.mlp.out.weight.std().item() < 0.02 / math.sqrt(2 * 2) * 1.5
    idx, tgt = _batch()
    _, loss = m(idx, tgt)
    loss.backward()
    assert torch.isfinite(loss) and all(p.grad is not None for p in m.parameters())

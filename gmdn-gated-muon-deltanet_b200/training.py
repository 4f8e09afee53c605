"""Config-4 training step: the ablation language model on the B200 mixer ops,
data-parallel over NCCL, with the outer Muon optimizer.

What it reproduces from the reference (train_ablation.py):

* the model: token embedding, ``n_layers`` pre-norm blocks (RMSNorm, the
  fast-weight mixer, RMSNorm, a 4x GELU MLP), final RMSNorm and an output head
  tied to the embedding (``Block``/``LM``, train_ablation.py:197-246), with the
  reference's initialisation (normal 0.02, residual output projections at
  0.02 / sqrt(2 L), the gate priors of train_ablation.py:102-109);
* the mixer: the same parameters as ``FastWeightMixer`` (train_ablation.py:
  84-110) whose forward is this library's prologue, chunk and epilogue ops
  (``integration.mixer_forward``);
* the optimisers: Nesterov Muon with Newton-Schulz msign on every 2-D hidden
  matrix and AdamW(0.9, 0.95) on the rest (train_ablation.py:60-73, 264-314);
* one step: bf16 autocast forward, cross-entropy on fp32 logits, backward,
  gradient clipping at 1.0, both optimiser steps (train_ablation.py:453-474),
  the learning-rate schedule and the evaluation pass (:310-314, 386-399);
* the run's records: the per-interval CSV and the incrementally rewritten
  JSON metrics file, and the final checkpoint, in the reference's formats
  (:426-444, 476-529), so its analysis scripts read them unchanged and its
  ``LM`` loads the checkpoint (same state-dict names).

B200 choices: the mixer's scan runs on the tcgen05 kernels (dh 64 at
d_model 768 / 12 heads); the msign of the outer Muon stacks every matrix of
one shape into one batch, so each Newton-Schulz step is three batched GEMMs
(cuBLAS, fp32 with TF32 tensor cores as the reference's trainer enables)
instead of three GEMMs per matrix; data parallelism is torch DDP over the NCCL
backend, whose bucketed gradient all-reduce overlaps the backward.
"""

from __future__ import annotations

import json
import math
import os
from collections import defaultdict

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import integration

NS_COEF = (3.4445, -4.7750, 2.0315)   # train_ablation.py:67
GATE_PRIORS = (3.0, -1.0, 1.0, 2.0)   # alpha, beta, mu, nu (train_ablation.py:102-109)


class MixerLayer(nn.Module):
    """The fast-weight mixer with FastWeightMixer's parameters; forward on the
    B200 ops (prologue, chunk_fast_weight, head_rmsnorm)."""

    def __init__(self, d_model: int, n_heads: int, inner: str, chunk: int = 64,
                 ns_steps: int = 3):
        super().__init__()
        if inner not in ("delta", "muon", "adam") or d_model % n_heads:
            raise ValueError(f"bad mixer shape or rule: {d_model}/{n_heads} {inner}")
        self.h, self.dh = n_heads, d_model // n_heads
        self.inner, self.chunk, self.ns_steps = inner, chunk, ns_steps
        self.qkv = nn.Linear(d_model, 3 * d_model, bias=False)
        self.conv = nn.Conv1d(3 * d_model, 3 * d_model, 4, groups=3 * d_model, padding=3)
        self.n_gates = 4 if inner == "adam" else 3
        self.gates = nn.Linear(d_model, self.n_gates * n_heads, bias=True)
        self.norm = nn.RMSNorm(self.dh)
        self.out = nn.Linear(d_model, d_model, bias=False)
        self.last_gate_means: dict = {}
        self.set_gate_priors()

    def set_gate_priors(self) -> None:
        with torch.no_grad():
            bias = self.gates.bias.view(self.n_gates, self.h)
            for i in range(self.n_gates):
                bias[i].fill_(GATE_PRIORS[i])

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return integration.mixer_forward(self, x)


class SwiGLU(nn.Module):
    """out(silu(gate(x)) * up(x)) with a 4x hidden width: the MLP that the
    benchmark description of config 4 names.  The reference's trainer uses a
    GELU MLP (train_ablation.py:202-205), which stays the default; indexing
    [2] gives the residual output projection like the GELU Sequential."""

    def __init__(self, d_model: int):
        super().__init__()
        self.gate = nn.Linear(d_model, 4 * d_model, bias=False)
        self.up = nn.Linear(d_model, 4 * d_model, bias=False)
        self.out = nn.Linear(4 * d_model, d_model, bias=False)

    def __getitem__(self, i: int) -> nn.Module:
        return {0: self.gate, 2: self.out}[i]

    def forward(self, x):
        return self.out(F.silu(self.gate(x)) * self.up(x))


class Block(nn.Module):
    def __init__(self, d_model: int, n_heads: int, inner: str, chunk: int, ns_steps: int,
                 mixer_cls=MixerLayer, mlp: str = "gelu"):
        super().__init__()
        self.n1 = nn.RMSNorm(d_model)
        self.mixer = mixer_cls(d_model, n_heads, inner, chunk, ns_steps)
        self.n2 = nn.RMSNorm(d_model)
        if mlp == "gelu":
            self.mlp = nn.Sequential(nn.Linear(d_model, 4 * d_model, bias=False), nn.GELU(),
                                     nn.Linear(4 * d_model, d_model, bias=False))
        elif mlp == "swiglu":
            self.mlp = SwiGLU(d_model)
        else:
            raise ValueError(f"mlp must be 'gelu' or 'swiglu', got {mlp!r}")

    def forward(self, x):
        x = x + self.mixer(self.n1(x))
        return x + self.mlp(self.n2(x))


class LanguageModel(nn.Module):
    """Embedding, blocks, final norm, tied output head; ``forward(idx,
    targets)`` returns (logits, mean cross-entropy or None)."""

    def __init__(self, vocab: int, d_model: int, n_layers: int, n_heads: int, inner: str,
                 chunk: int = 64, ns_steps: int = 3, mixer_cls=MixerLayer, mlp: str = "gelu"):
        super().__init__()
        self.emb = nn.Embedding(vocab, d_model)
        self.blocks = nn.ModuleList(Block(d_model, n_heads, inner, chunk, ns_steps, mixer_cls, mlp)
                                    for _ in range(n_layers))
        self.norm_f = nn.RMSNorm(d_model)
        self.lm_head = nn.Linear(d_model, vocab, bias=False)   # the reference's name
        self.lm_head.weight = self.emb.weight
        for m in self.modules():
            if isinstance(m, (nn.Linear, nn.Embedding)):
                nn.init.normal_(m.weight, std=0.02)
                if getattr(m, "bias", None) is not None:
                    nn.init.zeros_(m.bias)
        resid_std = 0.02 / math.sqrt(2 * n_layers)
        for blk in self.blocks:
            nn.init.normal_(blk.mixer.out.weight, std=resid_std)
            nn.init.normal_(blk.mlp[2].weight, std=resid_std)
            blk.mixer.set_gate_priors()

    def forward(self, idx, targets=None):
        x = self.emb(idx)
        for blk in self.blocks:
            x = blk(x)
        logits = self.lm_head(self.norm_f(x))
        if targets is None:
            return logits, None
        loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]).float(), targets.reshape(-1))
        return logits, loss

    def gate_means(self) -> dict:
        """Mean gate value per gate over the layers' last forward
        (train_ablation.py:248-257); NaN for a gate no layer reported."""
        vals = {k: [] for k in ("alpha", "beta", "mu", "nu")}
        for blk in self.blocks:
            for k in vals:
                v = blk.mixer.last_gate_means.get(k, float("nan"))
                v = v.item() if torch.is_tensor(v) else v
                if v == v:
                    vals[k].append(v)
        return {k: (sum(v) / len(v) if v else float("nan")) for k, v in vals.items()}


def msign(mats: torch.Tensor, steps: int = 5, eps: float = 1e-7) -> torch.Tensor:
    """Newton-Schulz orthogonalisation of a stack of matrices (..., r, c), in
    fp32 (train_ablation.py:60-73): tall matrices are handled transposed, each
    is divided by its Frobenius norm + eps, then ``steps`` quintic steps
    X <- a X + (b A + c A^2) X with A = X X^T.  The stack is one batch, so a
    step is three batched GEMMs whatever the number of matrices."""
    a, b, c = NS_COEF
    x = mats.float()
    tall = x.shape[-2] > x.shape[-1]
    if tall:
        x = x.mT
    x = x / (torch.linalg.matrix_norm(x, keepdim=True) + eps)
    for _ in range(steps):
        g = x @ x.mT
        p = torch.baddbmm(g, g, g, beta=b, alpha=c) if g.dim() == 3 else b * g + c * (g @ g)
        x = a * x + p @ x
    if tall:
        x = x.mT
    return x.to(mats.dtype)


class OuterMuon(torch.optim.Optimizer):
    """Nesterov-momentum Muon on 2-D matrices (train_ablation.py:264-288):
    buf <- m buf + g; u = g + m buf (Nesterov) or buf; u <- msign(u);
    p <- p (1 - lr wd) - lr sqrt(max(1, rows / cols)) u.  Parameters of one
    shape are orthogonalised together (one batched msign per shape)."""

    def __init__(self, params, lr=0.02, momentum=0.95, nesterov=True, weight_decay=0.0,
                 ns_steps=5):
        super().__init__(params, dict(lr=lr, momentum=momentum, nesterov=nesterov,
                                      weight_decay=weight_decay, ns_steps=ns_steps))

    @torch.no_grad()
    def step(self, closure=None):
        for group in self.param_groups:
            lr, mom, wd = group["lr"], group["momentum"], group["weight_decay"]
            by_shape = defaultdict(list)
            for p in group["params"]:
                if p.grad is not None:
                    by_shape[tuple(p.shape)].append(p)
            for shape, ps in by_shape.items():
                updates = []
                for p in ps:
                    st = self.state[p]
                    if "buf" not in st:
                        st["buf"] = torch.zeros_like(p.grad)
                    buf = st["buf"]
                    buf.mul_(mom).add_(p.grad)
                    updates.append(p.grad.add(buf, alpha=mom) if group["nesterov"] else buf)
                u = msign(torch.stack(updates), group["ns_steps"])
                scale = max(1.0, shape[0] / shape[1]) ** 0.5
                for p, ui in zip(ps, u.unbind(0)):
                    if wd:
                        p.mul_(1 - lr * wd)
                    p.add_(ui, alpha=-lr * scale)


Muon = OuterMuon   # the reference's name


def build_optimizers(model: nn.Module, muon_lr=0.02, adam_lr=4e-4, weight_decay=0.1,
                     outer: str = "muon"):
    """Every 2-D parameter but the (tied) embedding is a hidden matrix: outer
    "muon" puts them on Muon and the rest on AdamW(0.9, 0.95); outer "adam"
    puts both groups on AdamW (train_ablation.py:291-307)."""
    if outer not in ("muon", "adam"):
        raise ValueError(f"outer optimiser must be 'muon' or 'adam', got {outer!r}")
    base = model.module if hasattr(model, "module") else model
    emb = {id(base.emb.weight)}
    hidden, other = [], []
    for p in model.parameters():
        if p.requires_grad:
            (hidden if p.ndim == 2 and id(p) not in emb else other).append(p)
    adamw = dict(lr=adam_lr, betas=(0.9, 0.95), weight_decay=weight_decay)
    if outer == "muon":
        return [OuterMuon(hidden, lr=muon_lr, weight_decay=weight_decay),
                torch.optim.AdamW(other, **adamw)]
    return [torch.optim.AdamW(hidden, **adamw), torch.optim.AdamW(other, **adamw)]


def lr_factor(step: int, warmup: int, total: int) -> float:
    """Linear warm-up to 1 over ``warmup`` steps, then a cosine from 1 to 0.1
    at ``total`` (train_ablation.py:310-314)."""
    if step < warmup:
        return (step + 1) / warmup
    prog = (step - warmup) / max(1, total - warmup)
    return 0.1 + 0.9 * 0.5 * (1 + math.cos(math.pi * min(prog, 1.0)))


class LrSchedule:
    """Scales every parameter group's learning rate by ``lr_factor`` of the
    step, from the rates the groups had when it was built, as the reference's
    loop does before each step (train_ablation.py:453-457)."""

    def __init__(self, optimizers, warmup: int = 500, total: int = 9600):
        self.optimizers, self.warmup, self.total = optimizers, warmup, total
        self.base = [[g["lr"] for g in o.param_groups] for o in optimizers]

    def set_step(self, step: int) -> float:
        fac = lr_factor(step, self.warmup, self.total)
        for opt, bases in zip(self.optimizers, self.base):
            for g, b in zip(opt.param_groups, bases):
                g["lr"] = b * fac
        return fac


def train_step(model: nn.Module, optimizers, idx: torch.Tensor, targets: torch.Tensor,
               amp: bool = True) -> torch.Tensor:
    """One optimisation step (train_ablation.py:458-474 with accum = 1): bf16
    autocast forward, backward (under DDP the NCCL all-reduce of the gradient
    buckets overlaps it), clipping at 1.0, both optimiser steps.  Returns the
    loss (a device tensor; nothing synchronises the host)."""
    for opt in optimizers:
        opt.zero_grad(set_to_none=True)
    with torch.autocast(device_type="cuda", dtype=torch.bfloat16, enabled=amp):
        _, loss = model(idx, targets)
    loss.backward()
    torch.nn.utils.clip_grad_norm_(model.parameters(), 1.0)
    for opt in optimizers:
        opt.step()
    return loss.detach()


@torch.no_grad()
def evaluate(model: nn.Module, val_batches, amp: bool = True):
    """Mean loss over fixed validation batches and its perplexity
    exp(min(loss, 20)) (train_ablation.py:386-399); the model is left in
    training mode."""
    model.eval()
    total, n = 0.0, 0
    for x, y in val_batches:
        with torch.autocast(device_type="cuda", dtype=torch.bfloat16,
                            enabled=amp and x.is_cuda):
            _, loss = model(x, y)
        total += loss.item()
        n += 1
    model.train()
    loss = total / max(n, 1)
    return loss, math.exp(min(loss, 20))


# Column order and number formats of the per-interval CSV (train_ablation.py:
# 426-428, 497-501): its readers parse these exact columns.
CSV_COLUMNS = ("step", "train_loss", "val_loss", "val_ppl", "lr_hidden", "grad_norm", "tok_s",
               "alpha", "beta", "mu", "nu", "elapsed_s")


class RunLog:
    """The records of one training condition, in the reference's formats:

    * ``<cond>.csv``: a header line, then one row per logging interval;
    * ``<cond>_metrics.json``: ``{"meta": ..., "log": [rows]}``, rewritten in
      full after every row through a temporary file and ``os.replace`` (a
      crash leaves the previous complete file), and once more with
      ``meta["final"]`` at the end (train_ablation.py:429-444, 502-519).
    """

    def __init__(self, results_dir: str, condition: str, meta: dict):
        os.makedirs(results_dir, exist_ok=True)
        self.csv_path = os.path.join(results_dir, f"{condition}.csv")
        self.json_path = os.path.join(results_dir, f"{condition}_metrics.json")
        self.meta = dict(meta)
        self.rows: list = []
        with open(self.csv_path, "w") as f:
            f.write(",".join(CSV_COLUMNS) + "\n")

    def row(self, step: int, train_loss: float, val_loss: float, val_ppl: float,
            lr_hidden: float, grad_norm: float, tok_s: float, gates: dict, elapsed_s: float,
            tokens_seen: int) -> None:
        g = {k: gates.get(k, float("nan")) for k in ("alpha", "beta", "mu", "nu")}
        with open(self.csv_path, "a") as f:
            f.write(f"{step},{train_loss:.6f},{val_loss:.6f},{val_ppl:.4f},"
                    f"{lr_hidden:.6e},{grad_norm:.4f},{tok_s:.1f},"
                    f"{g['alpha']:.4f},{g['beta']:.4f},{g['mu']:.4f},"
                    f"{g['nu']:.4f},{elapsed_s:.1f}\n")
        self.rows.append(dict(
            step=step, train_loss=round(train_loss, 6), val_loss=round(val_loss, 6),
            val_ppl=round(val_ppl, 4), lr_hidden=lr_hidden, grad_norm=round(grad_norm, 4),
            tok_s=round(tok_s, 1), tokens_seen=tokens_seen,
            alpha=round(g["alpha"], 4), beta=round(g["beta"], 4), mu=round(g["mu"], 4),
            nu=round(g["nu"], 4), elapsed_s=round(elapsed_s, 1)))
        self.flush()

    def finish(self, result: dict) -> None:
        self.meta["final"] = dict(result)
        self.flush()

    def flush(self) -> None:
        tmp = self.json_path + ".tmp"
        with open(tmp, "w") as f:
            json.dump(dict(meta=self.meta, log=self.rows), f, indent=1)
        os.replace(tmp, self.json_path)


def save_checkpoint(path: str, model: nn.Module, *, vocab: int, d_model: int, n_layers: int,
                    n_heads: int, inner: str, chunk: int, outer: str, step: int, seed: int,
                    data_seed: int, args: dict, final_val_loss: float,
                    final_val_ppl: float) -> None:
    """``torch.save`` of the reference's checkpoint dictionary (train_ablation.py:
    516-528): the model's state dict under the reference's parameter names
    (``LM`` loads it), the model configuration, the condition and the run's
    arguments and final validation figures."""
    base = model.module if hasattr(model, "module") else model
    torch.save(dict(
        model_state=base.state_dict(),
        model_config=dict(vocab=vocab, d_model=d_model, n_layers=n_layers, n_heads=n_heads,
                          inner=inner, chunk=chunk),
        condition=f"outer-{outer}_inner-{inner}", outer=outer, inner=inner,
        step=step, seed=seed, data_seed=data_seed, args=dict(args),
        torch_version=torch.__version__,
        final_val_loss=final_val_loss, final_val_ppl=final_val_ppl,
    ), path)


def load_checkpoint(path: str, ns_steps: int = 3, map_location="cpu", mixer_cls=MixerLayer):
    """Rebuilds the model of a checkpoint written by ``save_checkpoint`` or by
    the reference's trainer and loads its weights; returns (model, checkpoint
    dictionary)."""
    ck = torch.load(path, map_location=map_location, weights_only=False)
    cfg = ck["model_config"]
    model = LanguageModel(cfg["vocab"], cfg["d_model"], cfg["n_layers"], cfg["n_heads"],
                          cfg["inner"], chunk=cfg["chunk"], ns_steps=ns_steps, mixer_cls=mixer_cls)
    model.load_state_dict(ck["model_state"])
    return model, ck

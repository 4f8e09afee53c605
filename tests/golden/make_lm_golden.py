"""Generate the fixture that pins the config-4 model and its checkpoint format
to the reference's trainer.

Run in the development container, where the reference checkout is readable:

    python tests/golden/make_lm_golden.py --ref <path-to-reference-checkout>

It imports the reference's ``train_ablation.py`` unmodified and records, on
CPU in float32, for each inner rule (delta, muon, adam): the state dict of a
small seeded ``LM`` (vocab 61, d_model 64, 2 layers, 2 heads of 32, chunk 32; the
reference's own initialisation and gate priors), a token batch, the logits and
loss of ``LM.forward`` on it (the eager fast_scan path), and the layers' gate
means.  tests/test_training.py loads these weights into this package's
``LanguageModel`` (same parameter names) and checks the same logits; the GPU
box never needs the reference.
"""

from __future__ import annotations

import argparse
import os
import sys

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference checkout (train_ablation.py)")
    args = ap.parse_args()
    sys.path.insert(0, os.path.abspath(args.ref))
    import train_ablation as ta   # the reference, unmodified

    out = {}
    for inner in ("delta", "muon", "adam"):
        torch.manual_seed(0)
        model = ta.LM(61, 64, 2, 2, inner, chunk=32, ns_steps=3)
        idx = torch.randint(0, 61, (2, 65), generator=torch.Generator().manual_seed(1))
        with torch.no_grad():
            logits, loss = model(idx[:, :-1], idx[:, 1:])
        out[inner] = dict(
            state={k: v.clone() for k, v in model.state_dict().items()},
            idx=idx, logits=logits, loss=loss, gate_means=model.gate_means())
    path = os.path.join(HERE, "lm.pt")
    torch.save(out, path)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


if __name__ == "__main__":
    main()

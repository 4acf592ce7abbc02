"""Generates the committed golden fixtures of tests/golden/ (run here only).

Sources (read from the mounted reference, never copied):
  * examples/custom_pytorch/run.py:43-50 `reference()` -- the reference's own
    independent FP32/FP16-boundary host implementation of the sparse INT4
    SwiGLU MLP. It calls `.cuda()`; for fixture generation that call is
    redirected to the CPU tensor itself (the arithmetic is unchanged).
  * predictor/predictor_cpu.cpp `ls_predict`, compiled unmodified into
    oracle/_ref/libls_predictor_ref.so by oracle/Makefile.

    python tests/golden/make_golden.py

Writes:
  reference_mlp.npz   run.py reference() outputs for toy groups (G = 2)
  config1.json        seed-0 config-1 selection from ls_predict + oracle y
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
# the reference checkout: $LEANSTREAM_REFERENCE, else `reference` beside the repository root
REFERENCE = Path(os.environ.get("LEANSTREAM_REFERENCE") or (ROOT.parent / "reference")).resolve()
sys.path.insert(0, str(ROOT))


def reference_cases():
    import torch

    sys.path.insert(0, str(REFERENCE))
    sys.path.insert(0, str(REFERENCE / "examples" / "custom_pytorch"))
    import run  # examples/custom_pytorch/run.py

    saved = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *a, **k: self  # CPU evaluation of the same arithmetic
    try:
        cases = {}
        # (name, q-range, x-scale, multiplier, selected, seed)
        specs = [
            ("toy_mult1", (-3, 4), 0.1, 1.0, [0, 1, 2, 5, 7], 11),
            ("toy_mult2", (-3, 4), 0.1, 2.0, [0, 1, 2, 5, 7], 11),
            ("full_range", (-8, 8), 0.05, 1.0, [6, 4, 3, 5], 5),
            ("negative_heavy", (-8, 1), 0.03, 1.0, [1, 2, 3, 4, 5, 6, 7], 9),
        ]
        for name, (lo, hi), xs, mult, sel, seed in specs:
            torch.manual_seed(seed)
            q = torch.randint(lo, hi, (8, 2, 3, 512), dtype=torch.int8)
            x = (torch.randn(512) * xs).half()
            y = run.reference(x, q, sel, mult)
            cases[name] = dict(q=q.numpy(), x=x.numpy(), selected=np.array(sel, np.int32),
                               multiplier=np.float32(mult), y=y.numpy())
        return cases
    finally:
        torch.Tensor.cuda = saved


def config1():
    from leanstream_b200.synthetic import make_layer, representative_rows
    from oracle import oracle as O

    L = make_layer(0, 1024, 64, 64)
    digest = hashlib.sha256(L.packed.tobytes() + L.scales.tobytes() + L.x.tobytes()).hexdigest()
    p = O.Predictor(64, 1024, 16, 1, 32)
    ids = p.predict(representative_rows(L), L.x.astype(np.float32))
    p.close()
    from leanstream_b200.synthetic import descriptors

    y16, _, _ = O.mlp(1024, 64, L.x, L.packed, L.scales, descriptors(ids))
    return dict(seed=0, hidden=1024, groups=64, group_size=64, k=16, input_sha256=digest,
                ids=[int(i) for i in ids], y_oracle_f16_hex=y16.view(np.uint16).tobytes().hex())


def main():
    cases = reference_cases()
    flat = {f"{name}/{k}": v for name, c in cases.items() for k, v in c.items()}
    np.savez_compressed(HERE / "reference_mlp.npz", **flat)
    (HERE / "config1.json").write_text(json.dumps(config1(), indent=1) + "\n")
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main()

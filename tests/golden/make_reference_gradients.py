"""Generate tests/golden/reference_gradients.{json,npz}: losses
``fold + lit (elementwise expression)`` compiled by the reference's front
end and lowered by remora_b200.autodiff to a value fold and one gradient map
per parameter; expected values and gradients from the reference's tape AD
(remora/ad.py:trace_via_tape_multi).  The first three losses and their
closed-form gradients are the reference's own GPU gradient tests
(remora/tests/test_ad_source.py:569-605).  Regenerate with:

    REMORA_REFERENCE=/path/to/remorac python tests/golden/make_reference_gradients.py
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
REF = os.environ.get("REMORA_REFERENCE", "/root/reference")
sys.path.insert(0, REF)
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(HERE))

from make_golden import specialise  # noqa: E402
from remora.ad import trace_via_tape_multi  # noqa: E402
from remora.runtime import _lambda_callable  # noqa: E402
from remora.types import FLOAT, ArrayType, StaticDim  # noqa: E402

from remora_b200.autodiff import compile_value_and_grad_source  # noqa: E402
from remora_b200.codegen import meta_record, spec_record  # noqa: E402

N = 8
VEC = ArrayType(FLOAT, (StaticDim(N),))
LOSSES = [
    ("polynomial", "(define/pi () (loss [x (Array Float 8)] Float) (fold + 0.0 (* (+ x 1.0) (- x 2.0))))", 1),
    ("cubic", "(define/pi () (loss [x (Array Float 8)] Float) (fold + 0.0 (* (* x x) x)))", 1),
    ("division", "(define/pi () (loss [x (Array Float 8)] Float) (fold + 0.0 (/ x (+ x 1.0))))", 1),
    ("exp_two_inputs", "(define/pi () (loss [x (Array Float 8) y (Array Float 8)] Float) "
                       "(fold + 0.5 (* (exp x) (- y (* x y)))))", 2),
    ("log_select", "(define/pi () (loss [x (Array Float 8)] Float) "
                   "(fold + 0.0 (map (lambda (v) (select (> v 1.0) (log v) (* v v))) x)))", 1),
]


def main() -> None:
    x = np.linspace(0.25, 2.0, N, dtype=np.float32)
    y = np.linspace(-1.0, 1.5, N, dtype=np.float32)
    records, arrays = [], {}
    for name, src, n in LOSSES:
        ptypes = (VEC,) * n
        module, metas = compile_value_and_grad_source(src, "loss", ptypes, name=f"remora_{name}")
        args = [x, y][:n]
        sp = specialise(src, "loss", list(ptypes), FLOAT)
        tape, idx = trace_via_tape_multi(sp.body, [a.astype(np.float64) for a in args], [p[0] for p in sp.params])
        adj = tape.reverse()
        grads = [np.asarray(adj[i], dtype=np.float64) for i in idx]
        try:
            arrays[f"{name}__value"] = np.asarray(_lambda_callable(sp, {})(*args), dtype=np.float64)
        except TypeError:  # the interpreter divides whole arrays with float(); no value to record
            arrays[f"{name}__value"] = np.asarray(np.nan)
        for k, a in enumerate(args):
            arrays[f"{name}__in{k}"] = a
            arrays[f"{name}__grad{k}"] = grads[k]
        records.append({"name": name, "source": src, "n_inputs": n,
                        "kernels": {m.name: {"spec": spec_record(module.kernels[m.name]), "meta": meta_record(m)}
                                    for m in metas}})
        print(name, [m.name for m in metas])
    # the reference's closed forms for its three GPU cases
    closed = {"polynomial": 2.0 * x - 1.0, "cubic": 3.0 * x * x, "division": 1.0 / ((x + 1.0) ** 2)}
    for name, g in closed.items():
        np.testing.assert_allclose(arrays[f"{name}__grad0"], g, rtol=1e-5, atol=1e-6)
        arrays[f"{name}__closed"] = g.astype(np.float32)
    (HERE / "reference_gradients.json").write_text(json.dumps(records, indent=1) + "\n")
    np.savez(HERE / "reference_gradients.npz", **arrays)


if __name__ == "__main__":
    main()

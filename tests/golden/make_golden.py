"""Generate tests/golden/golden.json and golden_rows.npz from the reference's
own kernels.

Run in a checkout next to the reference tree: it builds oracle/_ref/libtbref.so
from the reference sources (oracle/Makefile, REF_ROOT) and runs every case
through that library (impl=REF), i.e. through the reference's unmodified
tb_cpu_* functions.  Outputs are recorded as SHA-256 of the full result plus
the first 1024 values of the first and last rows; tests/test_oracle.py checks that the oracle restatement
reproduces every checksum bit-for-bit, and the GPU tests compare against the
sampled rows.  Inputs are regenerated from the seeds in workloads.py, so only
outputs are stored.

    python tests/golden/make_golden.py [REF_ROOT]

REF_ROOT defaults to $TB_REFERENCE_ROOT, else a checkout named `reference`
beside this repository.
"""
from __future__ import annotations

import hashlib
import json
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tensorbit-run_b200"))

from oracle import oracle as O  # noqa: E402
import workloads as W  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def cases():
    """(name, fn(impl) -> dict of named outputs); fn must be deterministic."""
    out = []
    mock = W.CONFIGS["mock"]
    li = W.layer_inputs(mock)
    emb = W.embedding_inputs(mock)
    lg = W.logits(mock)
    bf = O.f32_to_bf16

    out.append(("mock_res_rms_f32", lambda i: dict(zip(
        ("h", "y"), O.residual_rms_norm(li["x"], li["res"], li["gamma"], mock.eps, i)))))
    out.append(("mock_res_rms_bf16", lambda i: dict(zip(
        ("h", "y"), O.residual_rms_norm(bf(li["x"]), bf(li["res"]), bf(li["gamma"]), mock.eps, i)))))
    out.append(("mock_rms_f32", lambda i: {"y": O.rms_norm(li["x"], li["gamma"], mock.eps, i)}))
    out.append(("mock_silu_f32", lambda i: {"y": O.silu(li["gate"], i)}))
    out.append(("mock_gelu_f32", lambda i: {"y": O.gelu(li["gate"], i)}))
    out.append(("mock_swiglu_f32", lambda i: {"y": O.swiglu(li["gate"], li["up"], i)}))
    out.append(("mock_swiglu_bf16", lambda i: {"y": O.swiglu(bf(li["gate"]), bf(li["up"]), i)}))
    out.append(("mock_rope_f32", lambda i: dict(zip(
        ("q", "k"), O.rope(li["q"], li["k"], li["pos"], mock.theta, i)))))
    out.append(("mock_embedding_f32", lambda i: {"y": O.embedding(emb["ids"], emb["table"], i)}))
    out.append(("mock_softmax_f32", lambda i: {"y": O.softmax(lg, None, i)}))
    out.append(("mock_argmax_f32", lambda i: {"y": O.argmax(lg, i)}))

    big = W.CONFIGS["7b"]
    r = 32
    bi = W.layer_inputs(big, rows=r)
    out.append(("7b_res_rms_f32_32rows", lambda i: dict(zip(
        ("h", "y"), O.residual_rms_norm(bi["x"], bi["res"], bi["gamma"], big.eps, i)))))
    out.append(("7b_rope_f32_32rows", lambda i: dict(zip(
        ("q", "k"), O.rope(bi["q"], bi["k"], bi["pos"], big.theta, i)))))
    out.append(("7b_swiglu_f32_32rows", lambda i: {"y": O.swiglu(bi["gate"], bi["up"], i)}))
    blg = W.logits(big, rows=8)
    out.append(("7b_softmax_f32_8rows", lambda i: {"y": O.softmax(blg, None, i)}))
    out.append(("7b_argmax_f32_8rows", lambda i: {"y": O.argmax(blg, i)}))

    c70 = W.CONFIGS["70b"]
    l70 = W.logits(c70, rows=4)
    out.append(("70b_softmax_f32_4rows", lambda i: {"y": O.softmax(l70, None, i)}))
    r70 = W.layer_inputs(W.Config("70b_rows", 8, 8192, 64, 64, 8, 128, 128256, 5e5, 3.0, 4000,
                                  positions="uniform4096"))
    out.append(("70b_rope_f32_8rows", lambda i: dict(zip(
        ("q", "k"), O.rope(r70["q"], r70["k"], r70["pos"], 5e5, i)))))
    return out


def main():
    ref_root = (sys.argv[1] if len(sys.argv) > 1 else
                os.environ.get("TB_REFERENCE_ROOT",
                               os.path.join(os.path.dirname(ROOT), "reference")))
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "all", f"REF_ROOT={ref_root}"],
                   check=True, capture_output=True)
    O.lib()
    if not O.ref_available():
        raise SystemExit("oracle/_ref/libtbref.so missing: the reference tree is required")
    golden, rows = {}, {}
    for name, fn in cases():
        res = fn(O.REF)
        golden[name] = {k: {"sha256": sha(v), "shape": list(v.shape), "dtype": str(v.dtype)}
                        for k, v in res.items()}
        for k, v in res.items():
            # first and last row, first 1024 values of each (a spot check;
            # the checksum pins the whole output)
            flat = v.reshape(v.shape[0], -1) if v.ndim > 1 else v.reshape(1, -1)
            rows[f"{name}.{k}"] = flat[[0, -1], :1024]
        print(f"{name}: " + ", ".join(f"{k} {golden[name][k]['sha256'][:12]}" for k in res))
    meta = {"generator": "tests/golden/make_golden.py",
            "source": "reference src/ops/*.c compiled by oracle/Makefile (-O3 -mavx2 -mfma, gnu11)",
            "cases": golden}
    with open(os.path.join(HERE, "golden.json"), "w") as f:
        json.dump(meta, f, indent=1, sort_keys=True)
    np.savez_compressed(os.path.join(HERE, "golden_rows.npz"), **rows)


if __name__ == "__main__":
    main()

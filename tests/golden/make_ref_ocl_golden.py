"""Generates tests/golden/ref_ocl.npz from the reference's own OpenCL C kernels, compiled
unchanged for the host (oracle/_ref, built by oracle/ref_build.py from a reference checkout).

    python tests/golden/make_ref_ocl_golden.py

Cases (inputs stored beside the outputs, so the fixture does not depend on a libm):
  - gemm_q4_0_f16_portable on the two smallest shapes of crates/sulimo-ocl/tests/test_gemm.rs
    (N=8,K=256,M=256 and N=32,K=512,M=512) with that test's data generators;
  - kv_store_q8_0 on crates/sulimo-ocl/tests/test_prefill.rs:57-192's case (16 tokens x 8
    blocks, start_pos 5, capacity 64);
  - logits_f16_output on a seeded 96 x 256 Q4_0 matrix;
  - execute_prefill_ubatch on test_prefill.rs:296-566's 2-layer model and prompt (16 tokens):
    last-token logits, the final f16 residual stream and both layers' K/V rings.
tests/test_ref_pinning.py checks the C restatement (oracle/sulimo_oracle.c) against these
bit for bit, and against the live library where it is present.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.dirname(HERE))

import oracle.ffi as O  # noqa: E402
import oracle.ref_ffi as R  # noqa: E402
from helpers import (make_act_pattern_kv_store, make_model_pattern_prefill, make_q4_0,  # noqa: E402
                     make_q4_0_pattern_gemm, make_x_pattern_gemm, make_x_pattern_prefill)


def main():
    out = {}
    for tag, (n, k, m) in (("g0", (8, 256, 256)), ("g1", (32, 512, 512))):
        s, q = make_q4_0_pattern_gemm(m, k)
        x = make_x_pattern_gemm(n, k).view(np.uint16)
        out[f"{tag}_shape"] = np.array([n, k, m])
        out[f"{tag}_scales"], out[f"{tag}_quants"], out[f"{tag}_x"] = s, q, x
        out[f"{tag}_out"] = R.gemm_q4_0_f16_portable(s, q, x, m, k, n)

    act = make_act_pattern_kv_store(16, 8)
    kv = np.zeros(64 * 8 * 34, np.uint8)
    R.kv_store_q8_0(act, kv, 5, 64, 8, 16)
    out["kv_act"], out["kv_ring"] = act, kv

    s, q = make_q4_0(96, 256, seed=11)
    xs = np.random.default_rng(12).standard_normal(3 * 256).astype(np.float16).view(np.uint16)
    out["lg_scales"], out["lg_quants"], out["lg_x"] = s, q, xs
    out["lg_out"] = R.logits_f16_output(xs, s, q, 96, 256, 2)

    w = make_model_pattern_prefill()
    om = O.OracleModel(w)
    x0 = make_x_pattern_prefill(16, w["cfg"]["embd"])
    logits, x = R.execute_prefill_ubatch(om, np.zeros(16, np.int32), 0, x_f16=x0)
    out["pf_x0"], out["pf_logits"], out["pf_x"] = x0, logits, x
    for l, (kr, vr) in enumerate(om.rings):
        out[f"pf_k{l}"], out[f"pf_v{l}"] = kr, vr

    path = os.path.join(HERE, "ref_ocl.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()

"""Generates the golden fixtures under tests/golden/ from the REFERENCE itself.

Run once in a container that has the reference checkout (it is not needed at
test time and does not exist on the GPU hosts):

    python tests/golden/gen_golden.py [/path/to/llm-mojo]

What it writes
--------------
q4_golden.npz
    Seeded fp32 inputs and the packed nibbles + scales produced by the
    reference's own numpy quantizer, ``quantize_q4_0_vectorized`` in
    convert_gemma4_moe.py:9-35 (imported and executed here, unmodified).
    Cases cover N(0, 0.02) expert weights, N(0, 1), the 1e-5 scale floor,
    all-zero blocks, blocks whose max sits on an odd lane and a wide-range
    block.  Exact .5 rounding ties are excluded on purpose (numpy rounds them
    to even; the Mojo ``round`` in moe_kernels.mojo:46-47 is not pinned here),
    and the script asserts none remain.
known_answers.json
    Known-answer cases transcribed from the reference's Mojo tests, which
    cannot run without a Mojo toolchain:
      * LOD routing: test_moe_lod_top_p.mojo:28-49
      * top-k ordering: test_kernels.mojo:3021-3053
      * set-cover piggyback/prune: test_set_cover_moe.mojo:24-118
softmax_golden.npz
    numpy softmax references in the style of test_kernels.mojo:490-517.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference_quantizer(ref_root: str):
    sys.path.insert(0, ref_root)
    try:
        from convert_gemma4_moe import quantize_q4_0_vectorized  # noqa: E402
    finally:
        sys.path.pop(0)
    return quantize_q4_0_vectorized


def has_tie(x: np.ndarray) -> bool:
    b = x.reshape(-1, 32)
    scale = np.maximum(np.abs(b).max(1) / np.float32(7.0), np.float32(1e-5)).astype(np.float32)
    t = b * (np.float32(1.0) / scale)[:, None]
    return bool(np.any(np.abs(t - np.trunc(t)) == np.float32(0.5)))


def q4_cases(rng: np.random.Generator):
    cases = {}
    cases["expert_n002"] = rng.normal(0, 0.02, 8 * 2816).astype(np.float32)
    cases["unit_normal"] = rng.normal(0, 1, 4 * 704).astype(np.float32)
    cases["scale_floor"] = rng.normal(0, 1e-6, 64 * 32).astype(np.float32)
    z = rng.normal(0, 0.5, 32 * 32).astype(np.float32)
    z[5 * 32:6 * 32] = 0.0
    cases["zero_block"] = z
    oddmax = rng.normal(0, 0.1, 16 * 32).astype(np.float32)
    for b in range(16):
        oddmax[b * 32 + 2 * (b % 16) + 1] = np.float32(-0.9 if b % 2 else 0.9)
    cases["odd_lane_max"] = oddmax
    cases["wide_range"] = (rng.standard_normal(32 * 32) * np.exp(rng.uniform(-8, 4, 32 * 32))).astype(np.float32)
    return cases


def main(ref_root: str) -> None:
    quant = load_reference_quantizer(ref_root)
    rng = np.random.default_rng(20260601)
    out = {}
    for name, x in q4_cases(rng).items():
        # resample any block that would hit an exact .5 tie
        for _ in range(100):
            if not has_tie(x):
                break
            x = (x * np.float32(1.0000001)).astype(np.float32)
        assert not has_tie(x), name
        packed, scales = quant(x.copy())
        out[f"{name}__x"] = x
        out[f"{name}__packed"] = packed.astype(np.uint8)
        out[f"{name}__scales"] = scales.astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "q4_golden.npz"), **out)

    sm = {}
    for i, n in enumerate((16, 128, 128)):
        x = rng.standard_normal(n).astype(np.float32) * (1.0 if i < 2 else 8.0)
        e = np.exp(x - x.max())
        sm[f"case{i}__x"] = x
        sm[f"case{i}__p"] = (e / e.sum()).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "softmax_golden.npz"), **sm)

    known = {
        "lod": {
            "source": "test_moe_lod_top_p.mojo:28-49",
            "top_idx": [10, 25, 3, 77, 12, 99, 41, 8],
            "top_val": [0.42, 0.25, 0.15, 0.08, 0.04, 0.03, 0.02, 0.01],
            "expect_count_top_p_1": 4,
            "expect_count_top_p_080": 3,
            "expect_weight_sum_top_p_080": 1.0,
            "tol_weight_sum": 1e-5,
        },
        "top_k": {
            "source": "test_kernels.mojo:3021-3053",
            "probs": [1.0, 5.0, 2.0, 9.0, 0.5, 12.0, -1.0, 4.0, 3.0, 15.0, 6.0, 8.0, 0.1, 7.0, 11.0, 10.0],
            "expect_idx": [9, 5, 14, 15, 3, 11, 13, 10],
            "expect_val": [15.0, 12.0, 11.0, 10.0, 9.0, 8.0, 7.0, 6.0],
        },
        "set_cover": {
            "source": "test_set_cover_moe.mojo:24-118",
            "per_expert_scale": "0.8 + 0.4 * ((e * 17) % 31) / 31",
            "b0_idx": [10, 20, 30, 40, 50, 60, 70, 80],
            "b0_val": [0.28, 0.22, 0.16, 0.10, 0.07, 0.06, 0.06, 0.05],
            "bk_idx": "[10, 20, 30+b, 40, 50, 60, 90+2b, 91+2b]",
            "bk_val": [0.27, 0.23, 0.16, 0.12, 0.060, 0.055, 0.053, 0.052],
            "expect_count_b_ge_1": 6,
            "expect_renorm_sum": 1.0,
            "tol_renorm_sum": 1e-4,
        },
    }
    with open(os.path.join(HERE, "known_answers.json"), "w") as f:
        json.dump(known, f, indent=1)
    print("wrote", sorted(os.listdir(HERE)))


def _ref_dir() -> str:
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("LLM_MOJO_REF")
    if not ref:
        sys.exit("usage: gen_golden.py /path/to/llm-mojo  (or set LLM_MOJO_REF)")
    return ref


if __name__ == "__main__":
    main(_ref_dir())

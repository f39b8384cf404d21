"""Generates the golden fixtures in this directory from the C oracle.

    python tests/golden/make_golden.py

Each case uses seeded numpy inputs; outputs are what oracle/riallm_oracle.c
computes (a restatement of riallm's src/quantization.rs and
src/model.rs:751-818; parity with the Rust reference is unpinned because it
cannot run here). tests/test_oracle.py checks that the oracle still
reproduces these files bit for bit; the GPU tests compare the CUDA path
against them.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

QUANT_SIZES = [1, 2, 63, 64, 65, 127, 128, 129, 4095, 4096, 4097, 10000]

# (name, H, I, E, k, T, qtype, bf16, shared_I)
MOE_CASES = [
    ("moe_nf4_bf16", 256, 256, 4, 2, 5, O.FOUR_BIT, True, 0),
    ("moe_int8_bf16", 256, 256, 4, 2, 5, O.EIGHT_BIT, True, 0),
    ("moe_nf4_f32", 256, 256, 4, 2, 5, O.FOUR_BIT, False, 0),
    ("moe_nf4_bf16_k4_e8", 256, 256, 8, 4, 7, O.FOUR_BIT, True, 0),
    ("moe_nf4_bf16_shared", 256, 256, 4, 2, 3, O.FOUR_BIT, True, 256),
]


def quant_fixture():
    rng = np.random.default_rng(100)
    out = {}
    for n in QUANT_SIZES:
        v = rng.normal(0.0, 0.02, n).astype(np.float32)
        # sprinkle exact table values, zeros and out-of-range values
        if n >= 8:
            v[:8] = np.array([0.0, -0.0, 0.0150, -1.5, 2.0, 0.6962, -0.015, 0.0075], np.float32)
        out[f"v_{n}"] = v
        for name, qt in (("nf4", O.FOUR_BIT), ("int8", O.EIGHT_BIT)):
            t = O.quantize(v, qt)
            out[f"{name}_data_{n}"] = t.data
            out[f"{name}_scales_{n}"] = t.scales
            out[f"{name}_zeros_{n}"] = t.zero_points
            out[f"{name}_deq_{n}"] = O.dequantize(t)
    return out


def router_fixture():
    out = {}
    for (T, H, E, k, seed) in [(5, 256, 8, 2, 7), (9, 512, 128, 8, 8), (4, 1024, 8, 2, 9)]:
        rng = np.random.default_rng(seed)
        x = O.f32_to_bf16_bits(rng.normal(0, 1, (T, H)).astype(np.float32)).reshape(T, H)
        wg = rng.normal(0, 0.02, (E, H)).astype(np.float32)
        logits, probs, idx, w = O.router(x, wg, k)
        counts, offsets, perm = O.bucket(idx, E)
        tag = f"T{T}_H{H}_E{E}_k{k}"
        out.update({f"x_{tag}": x, f"wg_{tag}": wg, f"logits_{tag}": logits, f"probs_{tag}": probs,
                    f"idx_{tag}": idx, f"w_{tag}": w, f"counts_{tag}": counts,
                    f"offsets_{tag}": offsets, f"perm_{tag}": perm})
    return out


def moe_fixture(name, H, I, E, k, T, qt, bf16, shared_I, seed):
    w, _ = O.synthetic_layer(H, I, E, qt, seed, shared_intermediate=shared_I)
    x = O.synthetic_x(T, H, seed + 1, bf16=bf16)
    out, idx, tw, counts = O.moe_forward(w, x, T, H, I, E, k)
    d = {"x": x, "out": out, "idx": idx, "tw": tw, "counts": counts,
         "dims": np.array([H, I, E, k, T, qt, int(bf16), shared_I], np.int64)}
    names = ["gate", "gate_up_proj", "down_proj"]
    if shared_I:
        names += ["shared_gate_proj", "shared_up_proj", "shared_down_proj", "shared_expert_gate"]
    for n in names:
        t = getattr(w, n)
        d[f"{n}.qtype"] = np.array([t.qtype, t.block_size, t.numel], np.int64)
        d[f"{n}.data"] = t.data
        d[f"{n}.scales"] = t.scales
        d[f"{n}.zeros"] = t.zero_points
    return d


def main():
    np.savez_compressed(os.path.join(HERE, "quant.npz"), **quant_fixture())
    np.savez_compressed(os.path.join(HERE, "router.npz"), **router_fixture())
    for i, case in enumerate(MOE_CASES):
        name = case[0]
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **moe_fixture(*case, seed=200 + i))
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()

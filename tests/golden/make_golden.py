"""Generate the committed golden fixtures under tests/golden/.

    python tests/golden/make_golden.py

The inputs are the reference's own deterministic generators
(crates/sd-models/tests/mlx_quantized.rs:27-39: ``weight(out, in)`` and
``activation(rows, in)``) and its ``SeededRng`` (crates/sd-tensor/src/lib.rs:
104-145).  The outputs come from the CPU oracle (oracle/sdq_oracle.c), after
it has been checked bit for bit against the independent NumPy restatement in
oracle/oracle.py.  MLX itself cannot run here, so these pin the oracle's
rule (see oracle/sdq_oracle.h) rather than MLX's bits.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(HERE)), "oracle"))
import oracle as O  # noqa: E402


def edge_weight() -> np.ndarray:
    """[8, 128] f32 with one special case per group: constant, zeros of both signs, NaN
    and inf members, tiny and huge magnitudes, exact ties for round-half-even."""
    w = np.zeros((8, 128), np.float32)
    w[0, :64] = 0.25                                   # constant group (scale 0)
    w[0, 64:] = np.linspace(-1, 1, 64, dtype=np.float32)
    w[1, :64] = 0.0
    w[1, 1::2] = -0.0                                  # +0 / -0 only
    w[1, 64:] = np.float32(1e-30) * np.arange(64, dtype=np.float32)   # tiny
    w[2, :64] = np.arange(64, dtype=np.float32)        # exact integers 0..63
    w[2, 64:] = np.float32(3e38) * np.linspace(-1, 1, 64, dtype=np.float32)  # huge
    w[3, :64] = np.linspace(-2, 2, 64, dtype=np.float32)
    w[3, 5] = np.nan                                   # a NaN member
    w[3, 64:] = np.linspace(0, 1, 64, dtype=np.float32)
    w[3, 70] = np.inf                                  # an inf member
    w[4, :64] = np.nan                                 # all NaN
    w[4, 64:] = -np.arange(64, dtype=np.float32) / 7   # negative ramp
    w[5] = ((np.arange(128) % 3) - 1).astype(np.float32)  # {-1, 0, 1}
    w[6] = np.float32(0.5) + np.arange(128, dtype=np.float32) * np.float32(1.0 / 15.0)
    w[7] = np.float32(-1e-3) * np.arange(128, dtype=np.float32)
    return w


def main() -> None:
    O.build()
    out = {}
    w = O.reference_weight(256, 512)
    x = O.reference_activation(8, 512)
    xb = O.f32_to_bf16_bits(x)
    for bits in (4, 8):
        wq, s, b = O.quantize(w, bits)
        nq, ns, nb = O.np_quantize(w, bits)
        assert (wq == nq).all() and (s == ns).all() and (b == nb).all(), "C vs NumPy quantise"
        d = O.dequantize(wq, s, b, 256, 512, bits)
        assert (d == O.np_dequantize(wq, s, b, 256, 512, bits)).all(), "C vs NumPy dequantise"
        y = O.qmatmul(xb, wq, s, b, 256, bits)
        out[f"ref_b{bits}_wq"] = wq
        out[f"ref_b{bits}_scales"] = s
        out[f"ref_b{bits}_biases"] = b
        out[f"ref_b{bits}_dequant"] = d
        out[f"ref_b{bits}_qmm"] = y
    ew = edge_weight()
    for bits in (4, 8):
        wq, s, b = O.quantize(ew, bits)
        nq, ns, nb = O.np_quantize(ew, bits)
        assert (wq == nq).all() and (s == ns).all() and (b == nb).all(), "edge C vs NumPy"
        out[f"edge_b{bits}_wq"] = wq
        out[f"edge_b{bits}_scales"] = s
        out[f"edge_b{bits}_biases"] = b
        out[f"edge_b{bits}_dequant"] = O.dequantize(wq, s, b, 8, 128, bits)
    out["edge_w"] = ew
    out["rng_seed0_64"] = O.seeded_normals(0, 64)
    out["rng_seed42_65"] = O.seeded_normals(42, 65)
    np.savez_compressed(os.path.join(HERE, "quantized_linear.npz"), **out)
    print("wrote", os.path.join(HERE, "quantized_linear.npz"), sorted(out))


if __name__ == "__main__":
    main()

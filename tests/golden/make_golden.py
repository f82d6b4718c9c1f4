"""Generate golden KV-codec vectors from gguf-py (the reference's quantizer).

The reference converter calls ``gguf.quantize`` (convert_model_to_gguf.py:242-246)
and gguf-py's quants.py documents its Q8_0 as bit-exact with ggml-quants.c.
ggml itself is not available here, so gguf-py 0.19.0 is the pinned source of
truth for the KV block formats written by ggml_set_rows
(src/cosyvoice-kv-cache.cpp:316,322).

Run in the build container (gguf-py installed):
    python tests/golden/make_golden.py
Writes tests/golden/kv_codecs.npz.  The GPU box never runs this script; tests
read the committed .npz.
"""
from __future__ import annotations

import os

import numpy as np
import gguf
from gguf import GGMLQuantizationType as QT
from gguf import quants

HERE = os.path.dirname(os.path.abspath(__file__))
ROW = 128  # Hkv * D of the Qwen2 LLM KV rows (2 heads x 64)

TYPES = {
    "f32": QT.F32, "f16": QT.F16, "q8_0": QT.Q8_0, "q5_1": QT.Q5_1,
    "q5_0": QT.Q5_0, "q4_1": QT.Q4_1, "q4_0": QT.Q4_0,
}


def edge_rows(rng: np.random.Generator) -> np.ndarray:
    rows = []
    rows += list(rng.standard_normal((24, ROW)).astype(np.float32))
    # 1% outliers at +-8 sigma, as in the asymmetric-KV benchmark config
    x = rng.standard_normal((16, ROW)).astype(np.float32)
    hit = rng.random(x.shape) < 0.01
    x[hit] = np.where(rng.random(hit.sum()) < 0.5, -8.0, 8.0).astype(np.float32)
    rows += list(x)
    rows.append(np.zeros(ROW, np.float32))                           # all-zero blocks
    rows.append(np.full(ROW, -0.0, np.float32))                       # negative zeros
    z = np.zeros(ROW, np.float32); z[::7] = -0.0; z[3] = 1.0; rows.append(z)
    # exact rounding ties for Q8_0: amax = 127 gives d = 1, id = 1
    t = (np.arange(ROW, dtype=np.float32) % 120) - 60.0 + 0.5
    t[::32] = 127.0; t[5::32] = -126.5; rows.append(t.astype(np.float32))
    # Q4_0 / Q5_0 sign of the largest magnitude: -3 before +3 (first occurrence wins)
    s = rng.uniform(-1, 1, ROW).astype(np.float32); s[2::32] = -3.0; s[5::32] = 3.0; rows.append(s)
    s = rng.uniform(-1, 1, ROW).astype(np.float32); s[2::32] = 3.0; s[5::32] = -3.0; rows.append(s)
    rows.append(np.full(ROW, 0.75, np.float32))                        # constant blocks (d = 0 for _1 types)
    rows.append(np.full(ROW, -2.5, np.float32))
    rows.append((rng.standard_normal(ROW) * 1e-3).astype(np.float32))  # f16-subnormal scales
    rows.append((rng.standard_normal(ROW) * 1e-6).astype(np.float32))  # scales that flush to 0 in f16
    rows.append((rng.standard_normal(ROW) * 1e3).astype(np.float32))   # large values
    rows.append((rng.standard_normal(ROW) * 6e4).astype(np.float32))
    # f16 round-to-nearest-even midpoints and overflow (meaningful for the F16 type)
    m = np.full(ROW, 1.0, np.float32)
    m[0::4] = 1.0 + 2.0 ** -11; m[1::4] = 1.0 + 3 * 2.0 ** -11; m[2::4] = -(2.0 ** -25); m[3::4] = 2.0 ** -24 * 1.5
    rows.append(m)
    o = rng.standard_normal(ROW).astype(np.float32); o[0] = 70000.0; o[1] = -65520.0; o[2] = 65519.0
    rows.append(o)
    # one linearly increasing row per block to exercise every nibble / 5th bit
    rows.append(np.linspace(-4, 4, ROW, dtype=np.float32))
    return np.stack(rows).astype(np.float32)


def main() -> None:
    rng = np.random.default_rng(20261201)
    x = edge_rows(rng)
    out = {"x": x, "gguf_version": np.array(getattr(gguf, "__version__", "0.19.0"))}
    for name, qt in TYPES.items():
        data = x
        if name != "f16":
            # the F16 overflow row is only meaningful for F16; keep inputs finite in f16 range
            # for the block types too (gguf-py would store an inf scale otherwise)
            data = x.copy()
            data[-2, :3] = np.float32(1.0)
        q = quants.quantize(data, qt)
        q = np.ascontiguousarray(q).view(np.uint8).reshape(data.shape[0], -1)
        dq = quants.dequantize(q, qt).astype(np.float32).reshape(data.shape)
        out[f"{name}_x"] = data
        out[f"{name}_q"] = q
        out[f"{name}_dq"] = dq
    path = os.path.join(HERE, "kv_codecs.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {x.shape[0]} rows x {ROW} elements, types {list(TYPES)}")


if __name__ == "__main__":
    main()

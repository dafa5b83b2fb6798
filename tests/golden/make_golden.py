"""Generate the dequantization golden vectors under tests/golden/.

ggml's dequantize_row_q8_0 / _q4_K / _q6_K are the ground truth for the weight decode
(the reference calls them as ggml type traits' to_float, ggml-rocket.cpp:3894-3907).
ggml is not installed in the build container, so the vectors come from the `gguf`
Python package (version pinned below), whose `gguf.quants` module restates those
decoders in numpy. The inputs are random but valid blocks: random code bytes and
scale bytes, with the fp16 super-block scales drawn from a spread of finite exponents
(normal and subnormal), so that every bit of every field is exercised.

Run from the repository root:  python tests/golden/make_golden.py
"""
import os

import numpy as np

GGUF_VERSION = "0.19.0"

# block bytes and the byte offsets of each block's fp16 scale fields
LAYOUT = {
    "q8_0": dict(type_id=8, bytes=34, elems=32, f16_fields=[0]),
    "q4_k": dict(type_id=12, bytes=144, elems=256, f16_fields=[0, 2]),
    "q6_k": dict(type_id=14, bytes=210, elems=256, f16_fields=[208]),
}


def random_blocks(rng, n_blocks, spec):
    raw = rng.integers(0, 256, size=(n_blocks, spec["bytes"]), dtype=np.uint8)
    for off in spec["f16_fields"]:
        # finite fp16 magnitudes from 2^-24 (subnormal) to 2^3, both signs
        exp = rng.uniform(-24.0, 3.0, size=n_blocks)
        val = (np.sign(rng.standard_normal(n_blocks)) * np.exp2(exp)).astype(np.float16)
        val[0] = np.float16(0.0)   # one block with a zero scale
        raw[:, off:off + 2] = val.view(np.uint8).reshape(n_blocks, 2)
    return raw


def main():
    import gguf
    from gguf import quants

    import importlib.metadata
    assert importlib.metadata.version("gguf") == GGUF_VERSION
    out_dir = os.path.dirname(os.path.abspath(__file__))
    rng = np.random.default_rng(0xB200)
    classes = {"q8_0": quants.Q8_0, "q4_k": quants.Q4_K, "q6_k": quants.Q6_K}
    for name, spec in LAYOUT.items():
        n_blocks = 96
        raw = random_blocks(rng, n_blocks, spec)
        deq = classes[name].dequantize_blocks(raw.copy()).astype(np.float32).reshape(n_blocks, spec["elems"])
        # Q8_0 also from ggml's reference rounding, on N(0, 0.02) weights
        extra = {}
        if name == "q8_0":
            w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
            blocks = quants.Q8_0.quantize_blocks(w.reshape(-1, 32).astype(np.float32))
            extra = dict(q8_src=w, q8_quant=blocks.reshape(8, -1))
        np.savez_compressed(os.path.join(out_dir, f"dequant_{name}.npz"),
                            raw=raw, deq=deq, type_id=np.int32(spec["type_id"]),
                            gguf_version=np.array(GGUF_VERSION), **extra)
        print(f"{name}: {n_blocks} blocks -> dequant_{name}.npz")


if __name__ == "__main__":
    main()

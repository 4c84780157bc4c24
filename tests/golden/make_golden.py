"""Regenerates the reference's golden quant fixtures, byte for byte.

The reference commits runner/test/resources/fixtures/quants/<type>.safetensors
as Git LFS pointers only (sha256 + size); the bytes are not in its checkout.
Its generator, runner/fixtures/generate.py:41-91, draws them from
numpy.random.default_rng(42) -- 16 blocks per type in the order Q4_0, Q4_1,
Q5_0, Q5_1, Q8_0, Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, ..., block 0 all zeros, block 1 all 0xFF, the f16 scale
fields drawn as standard_normal * 0.05 -- and stores each block's decode by
gguf-py's `dequantize` as "expected".

This script follows that recipe with the installed gguf 0.19.0 (upstream
gguf-py; the reference pinned a fork at commit 9c37bc7, whose GGML types are
upstream's) and safetensors, and checks each file's sha256 against the LFS
pointer the reference commits (POINTERS below, copied from those pointer
files). A match means the committed fixtures ARE the reference's fixtures.

Run from the repo root:  python tests/golden/make_golden.py
"""

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# runner/test/resources/fixtures/quants/<name>.safetensors (Git LFS pointers):
# (oid sha256, size)
POINTERS = {
    "q4_0": ("53534083a9cfe19cdbe7e5b052dbaf215371b9608c70e168facd6af26e58b37b", 2480),
    "q4_1": ("ecf48132fc599e932c9dc438fdf6d53798bdf3bbc015ae17d7dd304aaafe6454", 2512),
    "q5_0": ("8208b9cfc49aa08a690a54a0b7e341d7c797bcda14ea1c946035827738665ca0", 2544),
    "q5_1": ("fdcf6eea0ba8968d7e5c25a3136cdce9bf66cce3c6c64eb0322065e290172d95", 2576),
    "q8_0": ("344260c8b28001cb9b2e7e78ef61e5e0cd59c9a6a6c1d99b87b181325c9109e0", 2736),
    "q2_k": ("bcc9580b7f5e838eb1958634d93e2a6119f1fde2f782232325f325509d28794a", 17880),
    "q3_k": ("c6367bd2af93905fd5fb6e8255faec578489bea1c20a47df651cc5bb1b946392", 18296),
    "q4_k": ("7f7f40d8244fb7b4918a075ecc6e1f58ecf257db487f3937a6a0130995e42912", 18840),
    "q5_k": ("c0227321921d000b342e0efd747e6c9cdb861bb7b594a4d0f5d9b72591fda899", 19352),
    "q6_k": ("073906d6b047810c6eff5d618bd43575357d57079973134db7024b18e5a188a4", 19896),
}
# the K-quants the library serves; the others are drawn only to keep the
# generator's random sequence
KEPT = {"q4_0", "q4_1", "q5_0", "q5_1", "q8_0", "q4_k", "q6_k"}


def generate() -> dict:
    from gguf import GGMLQuantizationType as T
    from gguf.quants import dequantize
    from safetensors.numpy import save

    random = np.random.default_rng(42)
    # (elements per block, bytes per block, offsets of the f16 fields), in the
    # generator's own order: the draws must come in the same sequence.
    layouts = [
        (T.Q4_0, 32, 18, [0]),
        (T.Q4_1, 32, 20, [0, 2]),
        (T.Q5_0, 32, 22, [0]),
        (T.Q5_1, 32, 24, [0, 2]),
        (T.Q8_0, 32, 34, [0]),
        (T.Q2_K, 256, 84, [80, 82]),
        (T.Q3_K, 256, 110, [108]),
        (T.Q4_K, 256, 144, [0, 2]),
        (T.Q5_K, 256, 176, [0, 2]),
        (T.Q6_K, 256, 210, [208]),
    ]
    count = 16
    files = {}
    for quant, elements, block_bytes, halves in layouts:
        blocks = random.integers(0, 256, size=(count, block_bytes), dtype=np.uint8)
        blocks[0] = 0
        blocks[1] = 0xFF
        for offset in halves:
            scales = (random.standard_normal(count) * 0.05).astype(np.float16)
            blocks[:, offset:offset + 2] = scales.view(np.uint8).reshape(count, 2)
        expected = dequantize(blocks.reshape(-1), quant).reshape(count, elements)
        files[quant.name.lower()] = save(
            {"blocks": blocks, "expected": expected.astype(np.float32)})
    return files


def main() -> int:
    files = generate()
    bad = 0
    for name, data in files.items():
        digest = hashlib.sha256(data).hexdigest()
        oid, size = POINTERS[name]
        ok = digest == oid and len(data) == size
        bad += not ok
        print(f"{name}: {len(data)} bytes, sha256 {'matches' if ok else 'DIFFERS from'} "
              f"the reference's LFS pointer")
        if name in KEPT:
            with open(os.path.join(HERE, "quants", f"{name}.safetensors"), "wb") as f:
                f.write(data)
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())

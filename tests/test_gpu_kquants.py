"""The K-quant products (Q4_K, Q6_K: tensor/KQuants.scala, the runner's
Q4_K / Q6_K matvec types, runner/kernels/matvec.hip:278-358) against the CPU
oracle's CpuLinear (decode by KQuants.element, Double sums), within the
benchmark's 1e-4 + 1e-3 |e| bar; the reference's golden super-blocks
(runner/test/resources/fixtures/quants/q4_k, q6_k) as weights, so every
code and both fixture blocks (all zeros, all ones) reach the kernel;
odd super-block counts per row (Q6_K rows 2-byte aligned); F32 and BF16 x;
1 to 40 rows of x (passes of 8)."""

import os

import numpy as np
import pytest
import torch

import oracle
from drift_b200 import synthetic
from drift_b200.ops import CudaOps, Stored
from tests.conftest import read_safetensors

pytestmark = pytest.mark.gpu

TYPES = {"q4_k": oracle.Q4_K, "q6_k": oracle.Q6_K}


@pytest.fixture(scope="module")
def ops():
    return CudaOps()


def check(ops, dtype, blocks, n, k, m, bf16, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((m, k)).astype(np.float32)
    if bf16:
        x = (x.view(np.uint32) & 0xFFFF0000).view(np.float32)  # exact in bf16
    w = Stored.upload(dtype, (n, k), blocks)
    xt = torch.from_numpy(x).cuda()
    if bf16:
        xt = xt.to(torch.bfloat16)
    y = torch.full((m, n), float("nan"), device="cuda")
    ops.linear(xt, w, y)
    got = y.cpu().numpy()
    expected = oracle.linear(dtype, x, blocks, n, k)
    bound = 1e-4 + 1e-3 * np.abs(expected)
    worst = float(np.max(np.abs(got - expected) - bound))
    assert np.all(np.abs(got - expected) <= bound), worst


@pytest.mark.parametrize("name", sorted(TYPES))
@pytest.mark.parametrize("m", [1, 3, 8])
def test_golden_blocks_as_weights(ops, golden_dir, name, m):
    """The reference's 16 fixture super-blocks as a [4, 1024] weight."""
    fixture = read_safetensors(os.path.join(golden_dir, "quants", f"{name}.safetensors"))
    blocks = fixture["blocks"].reshape(-1).copy()
    # scales drawn ~ N(0, 0.05) by the recipe: products of 1024 values stay
    # finite; the all-ones block's f16 fields are NaN-free by construction
    check(ops, TYPES[name], blocks, 4, 1024, m, False, m)


@pytest.mark.parametrize("name", sorted(TYPES))
@pytest.mark.parametrize("m,n,k,bf16", [(1, 4096, 4096, False), (1, 1000, 2816, False),
                                        (2, 512, 768, True), (8, 300, 4096, False),
                                        (9, 256, 1280, True), (40, 128, 512, False)])
def test_products_match_the_oracle(ops, name, m, n, k, bf16):
    dtype = TYPES[name]
    rng = np.random.default_rng(n + k + m)
    blocks = synthetic.k_quant_blocks(rng, dtype, n, k)
    check(ops, dtype, blocks, n, k, m, bf16, n * m)


def test_k_quant_refusals(ops):
    """Rows that are not whole super-blocks are refused, as DType.byteSize
    refuses them."""
    rng = np.random.default_rng(0)
    blocks = synthetic.k_quant_blocks(rng, oracle.Q4_K, 4, 512)
    w = Stored.upload(oracle.Q4_K, (4, 384), blocks)
    with pytest.raises(ValueError, match="not whole Q4_K blocks of 256"):
        ops.linear(torch.zeros(1, 384, device="cuda"), w, torch.empty(1, 4, device="cuda"))


def test_gguf_weights_feed_the_products(ops, tmp_path):
    """Q4_K, Q6_K and Q4_1 weights written by gguf-py's GGUFWriter, read by
    drift_b200.gguf and uploaded: the products equal the oracle's on the
    same bytes."""
    gguf_py = pytest.importorskip("gguf")
    from drift_b200 import gguf

    rng = np.random.default_rng(4)
    path = tmp_path / "weights.gguf"
    writer = gguf_py.GGUFWriter(str(path), "llama")
    raw = {}
    for name, dtype, quant, n, k in [("blk.0.ffn_up.weight", oracle.Q4_K, gguf_py.GGMLQuantizationType.Q4_K, 96, 1024),
                                     ("blk.0.ffn_down.weight", oracle.Q6_K, gguf_py.GGMLQuantizationType.Q6_K, 64, 768),
                                     ("output.weight", oracle.Q4_1, gguf_py.GGMLQuantizationType.Q4_1, 128, 512)]:
        blocks = (synthetic.k_quant_blocks(rng, dtype, n, k) if dtype != oracle.Q4_1
                  else synthetic.quantized(rng, dtype, n, k))
        writer.add_tensor(name, blocks.reshape(n, -1), raw_dtype=quant)
        raw[name] = (dtype, blocks, n, k)
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()
    f = gguf.open_file(str(path))
    for name, (dtype, blocks, n, k) in raw.items():
        t = f.tensors[name]
        assert t.dtype == dtype and t.shape == (n, k)
        w = f.upload(name)
        x = rng.standard_normal((3, k)).astype(np.float32)
        y = torch.empty(3, n, device="cuda")
        ops.linear(torch.from_numpy(x).cuda(), w, y)
        expected = oracle.linear(dtype, x, blocks, n, k)
        got = y.cpu().numpy()
        assert np.all(np.abs(got - expected) <= 1e-4 + 1e-3 * np.abs(expected)), name

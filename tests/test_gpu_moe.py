"""The whole mixture of a decode step in one launch (drift_moe_decode) against
the five launches it stands for -- the router product, the top-k, the routed
and shared experts' SwiGLU, their down products, the combine with the
residual and the next norm (with records) -- bit for bit in every output:
logits, ids, route weights, the experts' rows, the residual, the norm and
its records. C5's shape (512 experts, top-10, hidden 2048, expert rows of
512) and a small one; batches 1, 3 and 16; Q4_1, Q4_0 and Q8_0 weights."""

import numpy as np
import pytest
import torch

import oracle
from drift_b200 import synthetic
from drift_b200.ops import CudaOps, RowNorm, SharedExpert, Stored

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ops():
    return CudaOps()


def stored(rng, dtype, experts, n, k):
    return Stored.upload(dtype, (experts, n, k), synthetic.quantized(rng, dtype, experts * n, k))


@pytest.mark.parametrize("tokens", [1, 3, 16])
@pytest.mark.parametrize("experts,k,hidden,ffn,dtype", [
    (512, 10, 2048, 512, oracle.Q4_1), (16, 4, 256, 64, oracle.Q4_1),
    (64, 8, 1024, 256, oracle.Q4_0), (32, 6, 512, 128, oracle.Q8_0)])
def test_moe_launch_is_the_five_launches(ops, tokens, experts, k, hidden, ffn, dtype):
    rng = np.random.default_rng(tokens * 131 + experts + hidden)
    g = torch.Generator(device="cuda").manual_seed(tokens + experts)
    gate = stored(rng, dtype, experts + 1, ffn, hidden)
    up = stored(rng, dtype, experts + 1, ffn, hidden)
    down = stored(rng, dtype, experts + 1, hidden, ffn)
    router = 0.02 * torch.randn(experts, hidden, generator=g, device="cuda")
    shared_router = 0.02 * torch.randn(hidden, generator=g, device="cuda")
    norm_weight = 1 + 0.02 * torch.randn(hidden, generator=g, device="cuda")
    residual0 = torch.randn(tokens, hidden, generator=g, device="cuda")
    x0 = torch.randn(tokens, hidden, generator=g, device="cuda")
    slots = tokens * k + tokens

    def buffers():
        return dict(x=x0.clone(), residual=residual0.clone(),
                    logits=torch.full((tokens, experts), 7.0, device="cuda"),
                    ids=torch.full((slots,), -5, dtype=torch.int32, device="cuda"),
                    weights=torch.full((tokens, k), 7.0, device="cuda"),
                    gated=torch.full((slots, ffn), 7.0, device="cuda"),
                    out=torch.full((slots, hidden), 7.0, device="cuda"),
                    prepared=ops.prepared_x(tokens, hidden).fill_(0xA5))

    # the five launches (x's records from the post norm, as the step has them)
    a = buffers()
    ops.add_rms_norm(a["x"], None, RowNorm(torch.ones(hidden, device="cuda"), 1e-6, 0.0, a["x"]),
                     a["prepared"])
    b = {key: (value.clone() if key != "prepared" else value.clone()) for key, value in a.items()}
    a["ids"][tokens * k:] = experts
    route_ids = a["ids"][:tokens * k].view(tokens, k)
    ops.route_linear(a["x"], router, a["logits"], route_ids, a["weights"], a["prepared"])
    ops.experts_gated_linear(a["x"], gate, up, a["ids"], a["gated"], 0, a["prepared"],
                             shared_tail=True)
    ops.experts_linear(a["gated"], down, a["ids"], a["out"])
    ops.moe_combine_norm(a["out"][:tokens * k], a["weights"],
                         SharedExpert(a["out"][tokens * k:], a["x"], shared_router),
                         a["residual"], RowNorm(norm_weight, 1e-6, 0.0, a["x"]), a["prepared"])
    # the one launch
    ops.moe_decode(b["x"], b["prepared"], router, b["logits"], b["ids"], b["weights"], gate, up,
                   down, b["gated"], b["out"], shared_router, b["residual"],
                   RowNorm(norm_weight, 1e-6, 0.0, b["x"]), b["prepared"])
    torch.cuda.synchronize()
    assert ops.take_device_error() == 0
    for key in ("logits", "ids", "weights", "gated", "out", "residual", "x", "prepared"):
        assert torch.equal(a[key], b[key]), key

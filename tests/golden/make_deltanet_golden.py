"""Golden vectors for the Gated DeltaNet step, from the implementation the
reference restates: transformers' torch_causal_conv1d_update and
torch_recurrent_gated_delta_rule (models/qwen3_next/modeling_qwen3_next.py;
the reference's CpuSequence.gatedDeltaRule is "transformers'
torch_recurrent_gated_delta_rule, in double", ops/CpuSequence.scala:82).
transformers computes the rule in F32 whatever its inputs, so the vectors pin
the oracle to F32 precision, not to the bit.

    python tests/golden/make_deltanet_golden.py   # writes deltanet.npz beside it
"""

import os

import numpy as np
import torch
from transformers.models.qwen3_next.modeling_qwen3_next import (
    torch_causal_conv1d_update, torch_recurrent_gated_delta_rule)

HERE = os.path.dirname(os.path.abspath(__file__))


def main() -> None:
    rng = np.random.default_rng(2024)
    tokens, key_heads, value_heads, d, taps = 3, 2, 4, 32, 4
    channels = (2 * key_heads + value_heads) * d
    # the convolution: x [tokens, channels], weight [channels, taps], state [taps - 1, channels]
    x = rng.standard_normal((tokens, channels)).astype(np.float32)
    weight = (0.5 * rng.standard_normal((channels, taps))).astype(np.float32)
    conv_state = rng.standard_normal((taps - 1, channels)).astype(np.float32)
    state_t = torch.from_numpy(conv_state.T.copy()).unsqueeze(0)           # [1, channels, span]
    conv_out = torch_causal_conv1d_update(torch.from_numpy(x.T.copy()).unsqueeze(0), state_t,
                                          torch.from_numpy(weight), None, "silu")
    convolved = conv_out[0].T.contiguous().numpy()                           # [tokens, channels]
    conv_state_after = state_t[0].T.contiguous().numpy()
    # the rule on the convolved projections
    a = rng.standard_normal((tokens, value_heads)).astype(np.float32)
    b = rng.standard_normal((tokens, value_heads)).astype(np.float32)
    decay = (-np.exp(rng.uniform(-1.0, 1.5, value_heads))).astype(np.float32)  # -exp(A_log)
    dt_bias = rng.standard_normal(value_heads).astype(np.float32)
    state = (0.02 * rng.standard_normal((value_heads, d, d))).astype(np.float32)
    q = convolved[:, :key_heads * d].reshape(tokens, key_heads, d)
    k = convolved[:, key_heads * d:2 * key_heads * d].reshape(tokens, key_heads, d)
    v = convolved[:, 2 * key_heads * d:].reshape(tokens, value_heads, d)
    ratio = value_heads // key_heads
    tq = torch.from_numpy(q).repeat_interleave(ratio, dim=1).unsqueeze(0)
    tk = torch.from_numpy(k).repeat_interleave(ratio, dim=1).unsqueeze(0)
    tv = torch.from_numpy(v).unsqueeze(0)
    x_gate = torch.from_numpy(a) + torch.from_numpy(dt_bias)
    g = torch.from_numpy(decay) * torch.nn.functional.softplus(x_gate)
    beta = torch.sigmoid(torch.from_numpy(b))
    out, final = torch_recurrent_gated_delta_rule(tq, tk, tv, g.unsqueeze(0), beta.unsqueeze(0),
                                                  torch.from_numpy(state).unsqueeze(0), True,
                                                  use_qk_l2norm_in_kernel=True)
    np.savez(os.path.join(HERE, "deltanet.npz"), x=x, weight=weight, conv_state=conv_state,
             convolved=convolved, conv_state_after=conv_state_after, a=a, b=b, decay=decay,
             dt_bias=dt_bias, state=state, out=out[0].numpy(), state_after=final[0].numpy(),
             shape=np.array([tokens, key_heads, value_heads, d, taps]))


if __name__ == "__main__":
    main()

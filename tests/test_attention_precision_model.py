"""The arithmetic of the tcgen05 attention prefill (`attn_tc_kernel`,
mlx-lean-moe_b200/csrc/gdn_attention.cu), restated on the CPU and checked
against float64 causal softmax attention (`qw/attention.py:91-93`).

Per query row, keys in tiles of 64: scores S = q.k in float32 from bf16
inputs, in log2 units; the row's running maximum m moves (and O and the
running sum l are rescaled by 2^(m_old - m_new)) only when a tile's maximum
exceeds it by more than 8, so p = 2^(s - m) stays below 2^8; P is p rounded
to bf16, l sums the unrounded p, O += P V in float32; the result O / l is
rounded to bf16.  The lazy rescale rounds the row's dominant p to bf16 where
a rescale at every new maximum would have it at exactly 1, which costs
accuracy on peaked rows; after the output's own bf16 rounding the error must
stay within 1.4 times that of the exact result rounded to bf16.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import gdn_oracle as O

F = np.float32
LOG2E = 1.4426950408889634


def attention_model(Q, K, V, scale, rescale_bound=8.0, tile=64):
    L, HD = Q.shape
    sl2 = F(scale * LOG2E)
    S = (Q.astype(F) @ K.astype(F).T).astype(F)
    out = np.zeros((L, HD), F)
    for r in range(L):
        m, l = F(-np.inf), F(0)
        o = np.zeros(HD, F)
        for j0 in range(0, r + 1, tile):
            s = (S[r, j0:min(j0 + tile, r + 1)] * sl2).astype(F)
            mx = s.max()
            if mx > m + rescale_bound:
                if m != -np.inf:
                    a = F(np.exp2(m - mx))
                    o *= a
                    l *= a
                m = mx
            p = np.exp2(s - m).astype(F)
            l += p.sum(dtype=F)
            o += (O.bf16_round(p) @ V[j0:j0 + len(p)].astype(F)).astype(F)
        out[r] = o / l
    return O.bf16_round(out)


def exact_attention(Q, K, V, scale):
    Q, K, V = (a.astype(np.float64) for a in (Q, K, V))
    S = np.where(np.tril(np.ones((len(Q), len(K)), bool)), Q @ K.T * scale, -np.inf)
    P = np.exp(S - S.max(1, keepdims=True))
    return (P / P.sum(1, keepdims=True)) @ V


@pytest.mark.parametrize("sharpness", [1.0, 4.0, 12.0])
def test_lazy_rescale_keeps_the_bf16_output_close_to_the_rounded_exact_result(sharpness):
    rng = np.random.default_rng(3)
    L, HD = 400, 256
    Q = O.bf16_round(rng.standard_normal((L, HD)).astype(F) * sharpness)
    K = O.bf16_round(rng.standard_normal((L, HD)).astype(F))
    V = O.bf16_round(rng.standard_normal((L, HD)).astype(F))
    want = exact_attention(Q, K, V, HD ** -0.5)
    floor = O.rel_l2(O.bf16_round(want.astype(F)), want)
    got = O.rel_l2(attention_model(Q, K, V, HD ** -0.5), want)
    assert got <= 1.4 * floor, (got, floor)

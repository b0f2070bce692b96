"""Gated DeltaNet math: chunked form == recurrence (with initial state), conv state continuation,
affine state maps for the sequence-sharded CP chain."""

import math

import torch

from bridge_b200.ops.gdn import (causal_conv1d_reference, chunk_gated_delta_rule_reference,
                                 gated_delta_rule_recurrent)
from bridge_b200.parallel.gdn_state import affine_chunk_state_map


def _inputs(L=150, H=3, K=8, V=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(L, H, K, generator=g), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(L, H, K, generator=g), dim=-1)
    v = torch.randn(L, H, V, generator=g)
    gg = -torch.rand(L, H, generator=g) * 0.2
    beta = torch.rand(L, H, generator=g)
    h0 = torch.randn(H, K, V, generator=g) * 0.1
    return q, k, v, gg, beta, h0


def test_chunked_equals_recurrent_with_state():
    q, k, v, g, b, h0 = _inputs()
    o_ref, s_ref = gated_delta_rule_recurrent(q, k, v, g, b, h0, scale=1 / math.sqrt(8))
    o, s = chunk_gated_delta_rule_reference(q, k, v, g, b, [0, q.shape[0]], h0[None], scale=1 / math.sqrt(8),
                                            chunk_size=16)
    assert torch.allclose(o, o_ref, atol=1e-4) and torch.allclose(s[0], s_ref, atol=1e-4)


def test_split_continuation_equals_full():
    q, k, v, g, b, h0 = _inputs(L=100)
    o_full, s_full = gated_delta_rule_recurrent(q, k, v, g, b, h0, scale=0.3)
    o1, s1 = gated_delta_rule_recurrent(q[:37], k[:37], v[:37], g[:37], b[:37], h0, scale=0.3)
    o2, s2 = gated_delta_rule_recurrent(q[37:], k[37:], v[37:], g[37:], b[37:], s1, scale=0.3)
    assert torch.allclose(torch.cat([o1, o2]), o_full, atol=1e-5) and torch.allclose(s2, s_full, atol=1e-5)


def test_affine_state_map_composes_across_shards():
    q, k, v, g, b, h0 = _inputs(L=96)
    _, s_full = gated_delta_rule_recurrent(q, k, v, g, b, h0, scale=0.3)
    S = h0.clone()
    for a, e in ((0, 40), (40, 96)):
        M, C = affine_chunk_state_map(k[a:e], v[a:e], g[a:e], b[a:e], chunk_size=16)
        S = torch.matmul(M, S) + C
    assert torch.allclose(S, s_full, atol=1e-4)


def test_conv_state_continuation_and_dh0():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(20, 5, generator=g, requires_grad=True)
    w = torch.randn(5, 4, generator=g)
    y_full, st_full = causal_conv1d_reference(x, w, None, [0, 20], None)
    y1, st1 = causal_conv1d_reference(x[:7], w, None, [0, 7], None)
    y2, st2 = causal_conv1d_reference(x[7:], w, None, [0, 13], st1)
    assert torch.allclose(torch.cat([y1, y2]), y_full, atol=1e-6) and torch.allclose(st2, st_full, atol=1e-6)
    assert torch.all(st_full[:, :, 0] == 0)
    h0 = torch.randn(1, 5, 4, generator=g, requires_grad=True)
    y, _ = causal_conv1d_reference(x, w, None, [0, 20], h0)
    y[3:].sum().backward()      # rows >= W-1 never read the initial state
    assert torch.all(h0.grad == 0)

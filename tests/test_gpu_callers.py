"""GPU parity of the reference-facing callers of the prefill path:
``triton_kernel.semantic_block_attention_triton`` and
``reference.semantic_block_attention`` against the reference's own outputs,
``vllm_bridge.semantic_paged_attention`` and ``hf_patch.patch_model`` against
the oracle, and the explicit page-position path of ``paged_prefill``.

Tolerance (north star): atol 2e-3 / rtol 1e-2 (K / V pass through f16 pages).
"""

import numpy as np
import pytest
import torch

import inputs as gi
from oracle import prefill as op
from oracle import quant as oq

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
CASES = [("e2e_causal", gi.E2E_LAYOUT, (1, 2, 448, 64), 448, True),
         ("e2e_chunk", gi.E2E_LAYOUT, (2, 2, 16, 64), 448, False),
         ("partial_causal", gi.PREFILL_PARTIAL_LAYOUT, (2, 3, 100, 32), 100, True),
         ("gap_causal", gi.PREFILL_GAP_LAYOUT, (1, 2, 96, 32), 96, True),
         ("partial_causal_d128", gi.PREFILL_PARTIAL_LAYOUT, (1, 2, 100, 128), 100, True)]


def _layout(spec):
    from intent_attention import BlockLayout, BlockPolicy, SemanticBlock
    return BlockLayout([SemanticBlock(n, s, e, BlockPolicy[p], score=sc) for n, s, e, p, sc in spec])


def _inputs(i):
    name, spec, qshape, T_kv, causal = CASES[i]
    B, H, M, D = qshape
    q = gi.normal(600 + 3 * i, qshape)
    k = gi.normal(601 + 3 * i, (B, H, T_kv, D))
    v = gi.normal(602 + 3 * i, (B, H, T_kv, D))
    return name, spec, causal, q, k, v


@pytest.mark.parametrize("i", range(len(CASES)))
def test_semantic_block_attention_matches_reference(golden, i):
    from intent_attention.reference import semantic_block_attention
    name, spec, causal, q, k, v = _inputs(i)
    out, dbg = semantic_block_attention(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                                        torch.from_numpy(v).cuda(), _layout(spec), causal=causal, return_debug=True)
    ref = np.nan_to_num(golden("prefill_golden.npz")[name], nan=0.0)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=ATOL, rtol=RTOL)
    assert out.dtype == torch.float32
    assert dbg["selected_kv_tokens"] == op.selected_token_indices(spec).size


@pytest.mark.parametrize("i", range(len(CASES)))
def test_triton_entry_point_with_threshold_zero_matches_reference(golden, i):
    """With threshold 0 the GPU path's selection equals the exact-token path's
    on these layouts (every ATTEND block is scored)."""
    from intent_attention.triton_kernel import semantic_block_attention_triton
    name, spec, causal, q, k, v = _inputs(i)
    out = semantic_block_attention_triton(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(),
                                          torch.from_numpy(v).cuda(), _layout(spec), causal=causal, threshold=0.0)
    ref = np.nan_to_num(golden("prefill_golden.npz")[name], nan=0.0)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("use_quant", [False, True])
def test_triton_entry_point_threshold_and_quant(use_quant):
    """Default threshold 0.5 drops low ATTEND blocks; use_quant stores INT8
    pages with per-page, per-channel scales (64-token pages)."""
    from intent_attention.triton_kernel import semantic_block_attention_triton
    spec = gi.E2E_LAYOUT
    B, H, M, D, T = 2, 2, 192, 128, 448
    q, k, v = gi.normal(701, (B, H, M, D)), gi.normal(702, (B, H, T, D)), gi.normal(703, (B, H, T, D))
    out, dbg = semantic_block_attention_triton(torch.from_numpy(q).cuda().half(), torch.from_numpy(k).cuda().half(),
                                               torch.from_numpy(v).cuda().half(), _layout(spec), causal=True,
                                               return_debug=True, use_quant=use_quant)
    assert out.dtype == torch.float16
    assert dbg["selected_block_names"] == ["system", "doc_high", "recent"]
    kh, vh = (torch.from_numpy(x).half().float().numpy() for x in (k, v))
    sel = [s for s in spec if s[3] != "SKIP" and not (s[3] == "ATTEND" and (s[4] or 0) < 0.5)]
    if use_quant:
        PS = 64
        def q8(x):
            pages = x.reshape(B, H, T // PS, PS, D).reshape(-1, PS, D)
            return oq.quantize_pages(pages, "INT8", "channel")["recon"].reshape(B, H, T, D)
        kh, vh = q8(kh), q8(vh)
    ref = op.semantic_block_attention(torch.from_numpy(q).half().float().numpy(), kh, vh, sel, True)
    np.testing.assert_allclose(out.float().cpu().numpy(), np.nan_to_num(ref), atol=ATOL, rtol=RTOL)


@pytest.mark.parametrize("block_size", [16, 128])
@pytest.mark.parametrize("causal", [True, False])
def test_vllm_bridge(block_size, causal):
    from intent_attention.vllm_bridge import semantic_paged_attention
    g = np.random.default_rng(block_size + causal)
    H, D, NB = 4, 128, 40
    n_logical = 448 // block_size + (448 % block_size > 0)
    kc = g.standard_normal((NB, H, D, block_size)).astype(np.float32)
    vc = g.standard_normal((NB, H, D, block_size)).astype(np.float32)
    table = g.permutation(NB)[:n_logical].astype(np.int32)
    T = 24
    query = g.standard_normal((T, H, D)).astype(np.float32)
    spec = gi.E2E_LAYOUT
    out = semantic_paged_attention(torch.from_numpy(query).cuda().half(), torch.from_numpy(kc).cuda().half(),
                                   torch.from_numpy(vc).cuda().half(), torch.from_numpy(table), _layout(spec),
                                   block_size=block_size, causal=causal)
    kh = torch.from_numpy(kc).half().float().numpy()
    vh = torch.from_numpy(vc).half().float().numpy()
    qh = torch.from_numpy(query).half().float().numpy()
    ref = op.semantic_paged_attention(qh, kh, vh, table, spec, block_size, causal)
    np.testing.assert_allclose(out.float().cpu().numpy(), ref, atol=ATOL, rtol=RTOL)


def test_hf_patch_routes_sdpa_through_selected_blocks():
    import torch.nn as nn
    import torch.nn.functional as F
    from intent_attention.hf_patch import patch_model

    class Attention(nn.Module):
        def __init__(self, d=256, heads=2):
            super().__init__()
            self.heads = heads
            self.q_proj, self.k_proj = nn.Linear(d, d, bias=False), nn.Linear(d, d, bias=False)
            self.v_proj, self.o_proj = nn.Linear(d, d, bias=False), nn.Linear(d, d, bias=False)

        def forward(self, x):
            B, T, d = x.shape
            split = lambda t: t.view(B, T, self.heads, d // self.heads).transpose(1, 2)  # noqa: E731
            o = F.scaled_dot_product_attention(split(self.q_proj(x)), split(self.k_proj(x)), split(self.v_proj(x)))
            return self.o_proj(o.transpose(1, 2).reshape(B, T, d))

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = nn.ModuleList([Attention(), Attention()])

        def forward(self, x):
            for layer in self.layers:
                x = layer(x)
            return x

    torch.manual_seed(0)
    model = Model().cuda()
    x = torch.randn(1, 100, 256, device="cuda")
    layout = _layout(gi.PREFILL_PARTIAL_LAYOUT)
    with torch.no_grad():
        expect = x
        for layer in model.layers:
            B, T, d = expect.shape
            split = lambda t: t.view(B, T, 2, d // 2).transpose(1, 2).cpu().numpy()  # noqa: E731
            o = op.semantic_block_attention(split(layer.q_proj(expect)), split(layer.k_proj(expect)),
                                            split(layer.v_proj(expect)), gi.PREFILL_PARTIAL_LAYOUT, causal=False)
            o = torch.from_numpy(o).float().cuda().transpose(1, 2).reshape(B, T, d)
            expect = layer.o_proj(o)
        patch_model(model, lambda layer: layout if layer == 0 or layer == 1 else None, verbose=False)
        got = model(x)
    np.testing.assert_allclose(got.cpu().numpy(), expect.cpu().numpy(), atol=ATOL, rtol=RTOL)
    assert F.scaled_dot_product_attention.__module__.startswith("torch")


def test_page_positions_override():
    """Explicit per-slot positions give the same result as positions derived from bases."""
    from intent_attention import PagePool
    from intent_attention.paged import make_tag_map, paged_prefill
    g = np.random.default_rng(77)
    B, Ht, G, M, D, PS, W = 2, 2, 2, 64, 128, 16, 8
    NP = B * Ht * W
    k = torch.randn(NP, PS, D, device="cuda")
    pool = PagePool.allocate(NP, PS, D, ["F16"], "page", "cuda")
    pool.quantize_(k, -k, ["F16"] * NP)
    table = torch.arange(NP, dtype=torch.int32, device="cuda").view(B, Ht, W)
    pos = torch.from_numpy(g.permutation(W).astype(np.int32) * PS)[None, None, :].expand(B, Ht, W).contiguous().cuda()
    # the same pages listed so that page - base gives those positions
    bases = (torch.arange(B * Ht, dtype=torch.int32, device="cuda") * W).view(B, Ht)
    table2 = (bases[:, :, None] + pos // PS).to(torch.int32).contiguous()
    q = torch.randn(B, Ht * G, M, D, device="cuda", dtype=torch.bfloat16)
    qp = torch.arange(M, dtype=torch.int32, device="cuda")[None].expand(B, M).contiguous() + 40
    tags = torch.ones(NP, dtype=torch.uint8, device="cuda")
    tm = make_tag_map({1: "F16"})
    a = paged_prefill(q, pool, table2, None, tags, tm, q_positions=qp, bases=bases)
    # explicit positions: slot o of table2 holds page bases + pos/PS, so the same table with positions = pos
    b = paged_prefill(q, pool, table2, None, tags, tm, q_positions=qp, page_positions=pos)
    torch.cuda.synchronize()
    assert torch.equal(a, b)

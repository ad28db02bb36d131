"""Host-side contract of the drop-in modules (no GPU needed)."""

import numpy as np
import pytest
import torch

import intent_attention
from intent_attention import (AdaptiveFormatKernelConfig, AdaptivePageFormat, FusedDecodeConfig, FusedKVPrecision,
                              IntentQuantKernelConfig, TritonKVPrecision)
from intent_attention.fused_selected_quant_decode import fused_selected_quant_decode, metadata_to_kernel_tensors
from intent_attention import fused_selected_quant_decode as fsq_fn
from intent_attention.triton_adaptive_format_attention import make_adaptive_page_tables
from intent_attention.triton_intent_quant_attention import (fake_int8_pages_from_fp16, intent_quant_decode_attention_triton,
                                                            make_page_tables_from_selected_pages, make_precision_tensor)


def test_package_shadows_submodule_like_reference():
    # the package attribute is the function, the submodule stays importable
    assert callable(intent_attention.fused_selected_quant_decode)
    assert fsq_fn is fused_selected_quant_decode


def test_enum_values_and_configs():
    assert [int(x) for x in FusedKVPrecision] == [0, 1, 2]
    assert [int(x) for x in TritonKVPrecision] == [0, 1, 2, 3, 4, 5]
    assert [x.value for x in AdaptivePageFormat] == [0, 1, 2, 3]
    assert FusedDecodeConfig() == FusedDecodeConfig(16, 64, 64, 64)
    assert IntentQuantKernelConfig() == IntentQuantKernelConfig(16, 64, 64, 64)
    assert AdaptiveFormatKernelConfig().sparse_max_nnz == 256


@pytest.mark.parametrize("name", ["basic", "lossy", "empty", "trunc"])
@pytest.mark.parametrize("shape", [(1, 1, 64), (2, 3, 4)])
def test_metadata_to_kernel_tensors_cpu_matches_reference(golden, name, shape):
    g, metas = golden("fused_golden.npz"), golden("fused_metas.json")
    B, H, W = shape
    pt, prec, pc = metadata_to_kernel_tensors(metas[name], num_pages=12, B=B, H=H,
                                              config=FusedDecodeConfig(max_selected_pages=W))
    key = f"meta_{name}_{B}{H}{W}"
    np.testing.assert_array_equal(pt.numpy(), g[key + "_pt"])
    np.testing.assert_array_equal(prec.numpy(), g[key + "_prec"])
    np.testing.assert_array_equal(pc.numpy(), g[key + "_pc"])
    assert pt.dtype == prec.dtype == pc.dtype == torch.int32


def test_page_table_helpers_match_reference(golden):
    g = golden("triton_interp_golden.npz")
    ids, cnt = make_page_tables_from_selected_pages(torch.tensor([0, 2, 5], dtype=torch.int32), 2, 3, 8)
    np.testing.assert_array_equal(ids.numpy(), g["mk1_ids"]); np.testing.assert_array_equal(cnt.numpy(), g["mk1_cnt"])
    ids, cnt = make_page_tables_from_selected_pages(torch.arange(12, dtype=torch.int32).reshape(2, 3, 2), 2, 3, 4)
    np.testing.assert_array_equal(ids.numpy(), g["mk3_ids"]); np.testing.assert_array_equal(cnt.numpy(), g["mk3_cnt"])
    prec = make_precision_tensor(10, fp16_pages=torch.tensor([0, 1, 2]), int8_pages=torch.tensor([3, 4]))
    np.testing.assert_array_equal(prec.numpy(), g["prec_t"])
    ids, cnt = make_adaptive_page_tables(torch.tensor([3, 1, 2], dtype=torch.int32), 1, 1)
    np.testing.assert_array_equal(ids.numpy(), g["mka_ids"]); np.testing.assert_array_equal(cnt.numpy(), g["mka_cnt"])


def test_page_table_helper_errors():
    with pytest.raises(ValueError, match="exceeds max_selected_pages"):
        make_page_tables_from_selected_pages(torch.arange(10, dtype=torch.int32), 1, 1, 5)
    with pytest.raises(ValueError, match="must have shape"):
        make_page_tables_from_selected_pages(torch.zeros(2, 3, 2, 2, dtype=torch.int32), 2, 3)
    with pytest.raises(ValueError, match="must match batch and heads"):
        make_page_tables_from_selected_pages(torch.zeros(1, 3, 2, dtype=torch.int32), 2, 3)
    with pytest.raises(ValueError, match="exceeds max_selected_pages"):
        make_adaptive_page_tables(torch.arange(10, dtype=torch.int32), 1, 1, 5)
    with pytest.raises(ValueError):
        make_adaptive_page_tables(torch.zeros(2, 3, 4, 5), 2, 3)


def test_fake_int8_pages_match_reference(golden):
    g = golden("fused_golden.npz")
    import inputs as gi
    kf = torch.from_numpy(gi.normal(61, (8, 16, 64)).astype(np.float16))
    q, s = intent_attention.fused_selected_quant_decode.__globals__["fake_int8_pages_from_fp16"](kf)
    np.testing.assert_array_equal(q.numpy(), g["k_i8"])
    np.testing.assert_array_equal(s.numpy(), g["k_sc"])
    q, s = fake_int8_pages_from_fp16(torch.from_numpy(g["t6_pages"]))
    np.testing.assert_array_equal(q.numpy(), g["t6_q"])
    np.testing.assert_array_equal(s.numpy(), g["t6_sc"])
    assert s.dtype == torch.float32


def test_fused_decode_head_dim_error_precedes_device_check():
    q = torch.randn(2, 4, 1, 64, dtype=torch.float16)
    pages = torch.zeros(8, 16, 64, dtype=torch.float16)
    i8 = torch.zeros(8, 16, 64, dtype=torch.int8)
    sc = torch.ones(8)
    pt = torch.zeros(2, 4, 4, dtype=torch.int32)
    with pytest.raises(ValueError, match="head_dim"):
        fused_selected_quant_decode(q, pages, pages, i8, i8, sc, sc, pt, torch.zeros(8, dtype=torch.int32),
                                    torch.zeros(2, 4, dtype=torch.int32), FusedDecodeConfig(head_dim=128))


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-GPU behaviour")
def test_no_cpu_fallback():
    q = torch.randn(2, 4, 1, 64, dtype=torch.float16)
    pages = torch.zeros(8, 16, 64, dtype=torch.float16)
    i8 = torch.zeros(8, 16, 64, dtype=torch.int8)
    sc = torch.ones(8)
    pt = torch.zeros(2, 4, 4, dtype=torch.int32)
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_selected_quant_decode(q, pages, pages, i8, i8, sc, sc, pt, torch.zeros(8, dtype=torch.int32),
                                    torch.full((2, 4), 4, dtype=torch.int32))
    with pytest.raises(RuntimeError, match="Triton is not installed|CUDA is not available"):
        intent_quant_decode_attention_triton(q[:, :, 0], pages, pages, i8, i8, sc, sc,
                                             torch.zeros(2, 4, 64, dtype=torch.int32),
                                             torch.full((2, 4), 3, dtype=torch.int32), torch.zeros(20, dtype=torch.int32))

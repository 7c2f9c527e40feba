"""CPU-only checks of the C ABI library and of host-side validation.

No kernel is launched here: the library must load without a GPU, export every
entry point the header declares, and the Python layer must reject invalid
input (with the reference's error types) before anything reaches the device.
"""

import ctypes
import os
import re

import pytest
import torch

from flash_attn_b200 import _capi, flash_attn_func, flash_attn_varlen_func, store_kvcache
from flash_attn_b200 import vllm as fvllm
from flash_attn_b200.interface import MaskSpec

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                      "include", "flash_attn_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(fa_[a-z_0-9]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _capi.library()
    names = declared_functions()
    assert names, "no declarations parsed"
    for name in names:
        assert hasattr(lib, name), f"{name} missing from the shared library"
    assert set(names) == set(_capi.SIGNATURES), "ctypes signatures out of sync with the header"
    assert lib.fa_abi_version() == 2
    assert _capi.kernel_launches() >= 0


def test_library_build_id_matches_the_sources():
    # The library is a build artefact that travels beside the sources; its
    # embedded hash must describe exactly the sources checked out here.
    import build
    assert _capi.build_id() == build.source_hash(), (
        "the shared library was built from other sources; run `python flash-attn-mps_b200/build.py`")


def test_struct_layout_matches_header_order():
    # 19 tensor descriptors (80 bytes each), 13 4-byte scalars, then (ABI 2)
    # one more descriptor (8-byte aligned) and 2 scalars.
    assert ctypes.sizeof(_capi.Tensor) == 8 + 4 + 4 + 32 + 32
    head = (19 * 80 + 13 * 4 + 7) // 8 * 8
    assert ctypes.sizeof(_capi.AttentionArgs) == head + 80 + 8


def test_invalid_arguments_are_reported_without_a_gpu():
    lib = _capi.library()
    args = _capi.AttentionArgs()
    rc = lib.fa_attention_fwd(ctypes.byref(args), None)
    assert rc == _capi.FA_ERR_INVALID
    assert lib.fa_last_error().decode()


def test_reject_training_and_cpu_tensors():
    q = torch.randn(1, 2, 2, 16)
    with pytest.raises(NotImplementedError, match="dropout"):
        flash_attn_func(q, q, q, dropout_p=.1)
    with pytest.raises(ValueError, match="CUDA"):
        flash_attn_func(q, q, q)
    with pytest.raises(NotImplementedError):
        flash_attn_func(q.requires_grad_(), q, q)


def test_vllm_rejections_precede_launch():
    q = torch.randn(3, 4, 32)
    cu = torch.tensor([0, 3], dtype=torch.int32)
    base = dict(q=q, k=q[:, :2], v=q[:, :2], max_seqlen_q=3, cu_seqlens_q=cu, max_seqlen_k=3,
                cu_seqlens_k=cu)
    with pytest.raises(ValueError, match="fa_version"):
        fvllm.flash_attn_varlen_func(**base, fa_version=5)
    with pytest.raises(ValueError, match="cp_tot_seqused_k"):
        fvllm.flash_attn_varlen_func(**base, cp_world_size=2)
    with pytest.raises(NotImplementedError):
        fvllm.flash_attn_varlen_func(**base, q_v=q)
    with pytest.raises(NotImplementedError):
        fvllm.flash_attn_varlen_func(**base, output_scale=torch.ones(1))
    with pytest.raises(ValueError):
        fvllm.mm_prefix_mask(0)
    with pytest.raises(ValueError):
        fvllm.mm_prefix_mask(None, True)
    assert fvllm.rswa_mask() == MaskSpec(2)
    assert fvllm.get_scheduler_metadata(1, 2) is None


def test_store_validation():
    k = torch.randn(4, 2, 8)
    cache = torch.empty(2, 4, 2, 8)
    with pytest.raises(ValueError, match="CUDA"):
        store_kvcache(k, k, cache, cache, torch.zeros(4, dtype=torch.int64))


def test_paged_page_size_rule():
    q = torch.randn(3, 4, 32)
    k = torch.randn(2, 15, 2, 32)
    cu = torch.tensor([0, 3], dtype=torch.int32)
    with pytest.raises(ValueError, match="divisible by 16"):
        flash_attn_varlen_func(q, k, k, cu, cu, 3, 3, block_table=torch.zeros(1, 2, dtype=torch.int32))

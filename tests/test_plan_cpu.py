"""The decode split planner on the CPU, through the C ABI.

fa_attention_workspace_size only plans a call: it picks the kernel and the
split count from shapes, dtypes and features (never from device data) and
returns the bytes of split partials the call needs. It reads no memory, so the
descriptors here carry placeholder device addresses that are never touched.
The cases are the timed configurations of the benchmark -- config 4 (FP8 E4M3
paged decode, 64 x 131072 tokens, and one GPU's share at 8 GPUs), config 3
(bf16 paged decode, 256 ragged requests), the serving loop's decode step --
plus explicit split counts, the batch-invariant single split and the generic
kernel's rule (reference flash_attn_mps/_decode.py:63-64). The SM count falls
back to B200's 148 without a GPU, as on the GPU box.

Partials are fp32 [splits, T, Hq, Dv] and LSEs fp32 [splits, Hq, T], each
rounded up to 256 bytes; one split writes the output directly and needs none.
"""

import ctypes
import math

import pytest

from flash_attn_b200 import _capi

F16, BF16, F32, E4M3, I32 = 1, 2, 3, 4, 5
SIZE = {F16: 2, BF16: 2, F32: 4, E4M3: 1, I32: 4}
SMS = 148


class _Addresses:
    """Distinct, 4 KiB-aligned placeholder device addresses."""

    def __init__(self):
        self.next = 0x7F0000000000

    def tensor(self, dtype, shape):
        t = _capi.Tensor()
        t.ptr = self.next
        self.next += (SIZE[dtype] * math.prod(shape) // 4096 + 2) * 4096
        t.dtype, t.ndim = dtype, len(shape)
        stride = 1
        for i in reversed(range(len(shape))):
            t.shape[i], t.stride[i] = shape[i], stride
            stride *= shape[i]
        return t


def decode_args(batch, max_k, hq=32, hk=8, d=128, kv=BF16, q=BF16, page=16, splits=0, window=-1):
    mem = _Addresses()
    pages = -(-max_k // page)
    a = _capi.AttentionArgs()
    a.q, a.out = mem.tensor(q, [batch, hq, d]), mem.tensor(q if q != F32 else F32, [batch, hq, d])
    a.lse = mem.tensor(F32, [hq, batch])
    a.k = mem.tensor(kv, [batch * pages, page, hk, d])
    a.v = mem.tensor(kv, [batch * pages, page, hk, d])
    a.cu_seqlens_q = mem.tensor(I32, [batch + 1])
    a.seqused_k = mem.tensor(I32, [batch])
    a.block_table = mem.tensor(I32, [batch, pages])
    if kv == E4M3:
        a.k_descale, a.v_descale = mem.tensor(F32, [batch, hk]), mem.tensor(F32, [batch, hk])
    a.batch, a.max_seqlen_q, a.max_seqlen_k = batch, 1, max_k
    a.softmax_scale = d ** -0.5
    a.window_left, a.window_right = window, -1
    a.num_splits = splits
    a.cp_world_size = 1
    return a


def workspace(args):
    lib = _capi.library()
    n = ctypes.c_size_t()
    rc = lib.fa_attention_workspace_size(ctypes.byref(args), ctypes.byref(n))
    assert rc == 0, lib.fa_last_error().decode()
    return n.value


def partial_bytes(splits, tokens, hq, dv):
    if splits == 1:
        return 0
    up = lambda x: -(-x // 256) * 256  # noqa: E731
    return up(splits * tokens * hq * dv * 4) + up(splits * hq * tokens * 4)


def test_config4_fp8_decode_takes_four_splits():
    # FP8: at least 4 splits per (request, KV head); 64 x 8 units already give
    # ceil(8 * 148 / 512) = 3 < 4.
    assert workspace(decode_args(64, 131072, kv=E4M3)) == partial_bytes(4, 64, 32, 128)


def test_config4_shard_at_eight_gpus_keeps_four_splits():
    assert workspace(decode_args(64, 131072 // 8, kv=E4M3)) == partial_bytes(4, 64, 32, 128)


def test_fp8_small_batch_adds_splits_to_fill_the_gpu():
    # 8 requests x 8 KV heads = 64 units: ceil(8 * 148 / 64) = 19 splits.
    assert workspace(decode_args(8, 131072, kv=E4M3)) == partial_bytes(19, 8, 32, 128)


def test_fp8_splits_never_shorter_than_256_tokens():
    # by length: ceil(1000 / 256) = 4 caps the 19 the grid would want.
    assert workspace(decode_args(8, 1000, kv=E4M3)) == partial_bytes(4, 8, 32, 128)


def test_config3_bf16_decode_takes_four_splits():
    # 256 x 8 units >= 148 x 4 resident slots: 4 splits so that a ragged batch
    # does not end on its longest request.
    assert workspace(decode_args(256, 32768)) == partial_bytes(4, 256, 32, 128)


def test_serving_decode_step_runs_one_split():
    # Qwen3-0.6B-shaped serving loop: 64 requests x ~1152 tokens, 16 / 8 heads.
    # 512 units < 592 slots and 0.8 CTAs per slot need one split.
    assert workspace(decode_args(64, 1152, hq=16)) == 0


def test_bf16_few_requests_split_for_resident_grid():
    # 4 requests x 8 units = 32: ceil(0.8 * 592 / 32) = 15 splits.
    assert workspace(decode_args(4, 65536)) == partial_bytes(15, 4, 32, 128)


def test_window_limits_the_split_count():
    # A 300-token window leaves ceil(301 / 256) = 2 splits' worth of keys.
    assert workspace(decode_args(4, 65536, window=300)) == partial_bytes(2, 4, 32, 128)


@pytest.mark.parametrize("splits", [2, 8, 129])
def test_explicit_split_counts(splits):
    assert workspace(decode_args(64, 131072, kv=E4M3, splits=splits)) == partial_bytes(splits, 64, 32, 128)


def test_batch_invariant_single_split_needs_no_partials():
    assert workspace(decode_args(64, 131072, kv=E4M3, splits=1)) == 0


def test_fp32_decode_follows_the_generic_rule():
    # fp32 inputs run on the SIMT kernel with the reference's split rule
    # min(32, ceil(max_seqlen_k / 256)).
    assert workspace(decode_args(2, 4096, q=F32, kv=F32)) == partial_bytes(16, 2, 32, 128)
    assert workspace(decode_args(2, 131072, q=F32, kv=F32)) == partial_bytes(32, 2, 32, 128)

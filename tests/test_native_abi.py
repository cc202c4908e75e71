"""The C-ABI library loads without a GPU and exports what include/ declares (CPU only).

No kernel is launched here: only host-side entry points (version, status
strings, the decode plan, argument rejection) run.
"""

from __future__ import annotations

import ctypes
import os
import re

import pytest
import torch

import mini_vllm_b200 as M
from mini_vllm_b200 import _native

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include",
                      "mini_vllm_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(mvb_\w+)\s*\(", text, re.M)))


def test_header_declares_the_abi():
    syms = declared_symbols()
    assert "mvb_kv_cache_write" in syms and "mvb_paged_decode" in syms
    assert set(syms) == set(_native.SIGNATURES), "ctypes table and header must list the same symbols"


def test_library_exports_every_declared_symbol():
    lib = _native.lib()
    raw = ctypes.CDLL(_native.LIB_PATH)
    for name in declared_symbols():
        assert hasattr(raw, name), name
        assert hasattr(lib, name), name


def test_abi_version_and_status_strings():
    lib = _native.lib()
    assert lib.mvb_abi_version() == _native.ABI_VERSION
    assert "head_dim" in _native.status_string(_native.ERR_HEAD_DIM)
    assert "power of 2" in _native.status_string(_native.ERR_BLOCK_SIZE)
    assert _native.status_string(0) == "ok"
    assert _native.status_string(-999) == "unknown status"


def test_header_constants_match_binding():
    text = open(HEADER).read()
    consts = dict((k, int(v, 0)) for k, v in re.findall(r"#define\s+(MVB_\w+)\s+(-?(?:0x[0-9a-fA-F]+|\d+))", text))
    assert consts["MVB_DTYPE_BF16"] == _native.DTYPE_BF16
    assert consts["MVB_DTYPE_F16"] == _native.DTYPE_F16
    assert consts["MVB_DEV_DUP_SLOT"] == _native.DEV_DUP_SLOT
    assert consts["MVB_DEV_TIMEOUT"] == _native.DEV_TIMEOUT
    assert consts["MVB_ERR_VARIANT"] == _native.ERR_VARIANT
    assert consts["MVB_DECODE_MMA"] == _native.DECODE_MMA
    assert consts["MVB_DECODE_STREAM"] == _native.DECODE_STREAM
    assert consts["MVB_DECODE_AFTER_WRITE"] == _native.DECODE_AFTER_WRITE
    assert consts["MVB_DECODE_SCHED"] == _native.DECODE_SCHED
    assert consts["MVB_DECODE_SCHEDULE_READY"] == _native.DECODE_SCHEDULE_READY
    assert consts["MVB_DEV_SCHEDULE"] == _native.DEV_SCHEDULE


def _plan(**kw):
    args = dict(num_seqs=256, num_heads=14, num_kv_heads=2, head_dim=64, block_size=16,
                num_blocks=20000, max_blocks_per_seq=128, dtype=torch.bfloat16)
    args.update(kw)
    return M.decode_plan(**args)


def test_plan_headline_config_uses_the_stream_kernel():
    assert _plan()["variant"] == "stream"


def test_plan_auto_crossover_from_the_sweep():
    """AUTO follows the batch x context sweep: short contexts run one CTA per
    (sequence, KV head) unsplit, little work runs 512-token split-K, the rest
    streams (148 SMs without a GPU)."""
    short = _plan(num_seqs=64, max_blocks_per_seq=8)  # 128 tokens
    assert short["variant"] == "mma" and short["num_partitions"] == 1
    little = _plan(num_seqs=1, max_blocks_per_seq=512)  # 1 x 8192 tokens: 2 x 16 partitions
    assert little["variant"] == "mma" and little["partition_tokens"] == 512 and little["num_partitions"] == 16
    assert _plan(num_seqs=8, max_blocks_per_seq=512)["variant"] == "mma"  # 256 CTAs <= 2 x 148
    assert _plan(num_seqs=32, max_blocks_per_seq=512)["variant"] == "stream"  # 1024 CTAs
    assert _plan(num_seqs=5000, max_blocks_per_seq=128)["variant"] == "sched"  # past the stream kernel's batch limit


def test_plan_scheduled_kernel_when_asked():
    p = _plan(variant="sched")
    assert p["variant"] == "sched" and p["num_partitions"] == 0
    # header, a 256-byte record per CTA (148 SMs without a GPU), 512 units + 148
    # pieces, 512 units x 128 tiles of rows, 256 left-out slots, 148 counters,
    # and two partial states of 7 head rows x (64 + 4) floats per CTA
    import sched_model

    lay = sched_model.sched_layout(256, 2, 1, 128, 16, 148, G=7, head_dim=64)
    assert p["workspace_bytes"] == lay["bytes"]
    assert lay["bytes"] >= 256 + 148 * 256 + 660 * 32 + 65536 * 4 + 256 * 4 + 148 * 4 + 296 * 7 * 68 * 4


def test_plan_launches():
    """Kernels one decode call launches: the stream kernel + its fixup;
    split-K + its reduction; the scheduled kernel's schedule + decode."""
    assert _plan(variant="stream")["launches"] == 2
    assert _plan(variant="mma", partition_tokens=512)["launches"] == 2
    assert _plan(variant="mma")["launches"] == 1
    assert _plan(variant="sched")["launches"] == 2


def test_plan_stream_kernel_when_asked():
    p = _plan(variant="stream")
    assert p["variant"] == "stream" and p["num_partitions"] == 0
    # tile prefix + context lengths, then two partial slots (16 rows x (64 + 2) floats) per warp
    assert p["workspace_bytes"] >= (2 * 256 + 1) * 4 + 2 * 16 * 66 * 4 * 148


def test_plan_one_cta_per_sequence_and_kv_head_when_asked():
    p = _plan(variant="mma")
    assert p == {"variant": "mma", "partition_tokens": 2048, "num_partitions": 1, "workspace_bytes": 0, "launches": 1}


def test_plan_stream_limits():
    assert _plan(num_seqs=4096, variant="stream")["variant"] == "stream"
    assert _plan(num_seqs=4097)["variant"] == "sched"  # the scheduled kernel has no batch limit
    with pytest.raises(RuntimeError, match="variant"):
        _plan(num_seqs=4097, variant="stream")


def test_plan_long_context_uses_split_k():
    p = _plan(num_seqs=32, max_blocks_per_seq=2048, num_blocks=72090, variant="mma")
    assert p["variant"] == "mma" and p["partition_tokens"] == 512 and p["num_partitions"] == 64
    n = 32 * 14 * 64
    assert p["workspace_bytes"] >= n * 64 * 4 + 2 * n * 4


def test_plan_fp32_and_small_blocks_use_fma():
    assert _plan(dtype=torch.float32)["variant"] == "fma"
    assert _plan(block_size=8, max_blocks_per_seq=256)["variant"] == "fma"
    with pytest.raises(RuntimeError, match="variant"):
        _plan(dtype=torch.float32, variant="stream")
    with pytest.raises(RuntimeError, match="variant"):
        _plan(dtype=torch.float32, variant="mma")
    with pytest.raises(RuntimeError, match="variant"):
        _plan(block_size=8, max_blocks_per_seq=256, variant="sched")


def test_plan_explicit_partition_rounds_to_16():
    p = _plan(partition_tokens=100, variant="mma")
    assert p["partition_tokens"] == 112 and p["num_partitions"] == 19


@pytest.mark.parametrize("kw,match", [
    (dict(head_dim=96), "head_dim"),
    (dict(block_size=3), "power of 2"),
    (dict(num_heads=14, num_kv_heads=3), "multiple"),
])
def test_plan_rejects_bad_shapes(kw, match):
    with pytest.raises(AssertionError, match=match):
        _plan(**kw)


def test_kv_write_host_checks_without_gpu():
    lib = _native.lib()
    # zero tokens: nothing to do, no device touched
    assert lib.mvb_kv_cache_write(None, 0, 0, None, 0, 0, None, None, None, 0, 2, 64, 16, 4,
                                  _native.DTYPE_BF16, None, 0, None, None) == _native.OK
    assert lib.mvb_kv_cache_write(None, 0, 0, None, 0, 0, None, None, None, 1, 2, 64, 16, 4,
                                  7, None, 0, None, None) == _native.ERR_DTYPE
    assert lib.mvb_kv_cache_write(None, 0, 0, None, 0, 0, None, None, None, 1, 2, 64, 0, 4,
                                  _native.DTYPE_BF16, None, 0, None, None) == _native.ERR_BLOCK_SIZE
    assert lib.mvb_kv_cache_write(None, 0, 0, None, 0, 0, None, None, None, 1, 2, 64, 16, 4,
                                  _native.DTYPE_BF16, None, 0, None, None) == _native.ERR_INVALID_ARG


def test_decode_host_checks_without_gpu():
    lib = _native.lib()
    common = dict(bt_stride=8, maxb=8)

    def call(num_seqs, head_dim=64, block_size=16, nh=14, nkv=2, ws=None, wsb=0, variant=0, part=0):
        return lib.mvb_paged_decode(None, 0, 0, None, None, None, common["bt_stride"], common["maxb"], None,
                                    None, 0, 0, num_seqs, nh, nkv, head_dim, block_size, 100, 0.125,
                                    _native.DTYPE_BF16, variant, part, ws, wsb, None, None)

    assert call(0) == _native.OK  # empty batch
    assert call(1) == _native.ERR_INVALID_ARG  # null pointers
    assert call(1, head_dim=80) == _native.ERR_HEAD_DIM
    assert call(1, block_size=12) == _native.ERR_BLOCK_SIZE
    assert call(1, nh=7, nkv=2) == _native.ERR_HEADS


def test_schedule_host_checks_without_gpu():
    lib = _native.lib()

    def call(num_seqs, kv_len=None, bt=None, bt_stride=8, ws=None, wsb=0, flags=0, dtype=_native.DTYPE_BF16,
             err=None, variant=_native.DECODE_SCHED):
        return lib.mvb_paged_decode_schedule(kv_len, bt, bt_stride, num_seqs, 14, 2, 64, 16, 100, 8, dtype,
                                             variant, flags, ws, wsb, err, None)

    for v in (_native.DECODE_SCHED, _native.DECODE_STREAM):
        assert call(0, variant=v) == _native.OK  # empty batch: nothing launched
        assert call(1, variant=v) == _native.ERR_INVALID_ARG  # null kv_len
        assert call(1, kv_len=16, err=16, variant=v) == _native.ERR_INVALID_ARG  # null block table
        # rows shorter than 8 blocks
        assert call(1, kv_len=16, bt=16, bt_stride=4, err=16, variant=v) == _native.ERR_INVALID_ARG
        assert call(1, dtype=_native.DTYPE_F32, variant=v) == _native.ERR_VARIANT  # bf16 / f16 kernels only
        assert call(1, kv_len=16, bt=16, err=16, flags=0x400, variant=v) == _native.ERR_INVALID_ARG  # unknown flag
        assert call(1, kv_len=16, bt=16, err=16, variant=v) == _native.ERR_WORKSPACE  # no workspace
        # misaligned
        assert call(1, kv_len=16, bt=16, err=16, ws=256 * 7 + 16, wsb=1 << 30, variant=v) == _native.ERR_WORKSPACE
    # more sequences than the schedule kernel's prefix arrays hold: the plan refuses the variant
    assert call(16385, kv_len=16, bt=16, err=16) == _native.ERR_VARIANT
    assert call(4097, kv_len=16, bt=16, err=16, variant=_native.DECODE_STREAM) == _native.ERR_VARIANT
    # kernels without a per-step set-up: nothing to build, nothing launched
    assert call(1, kv_len=16, bt=16, err=16, variant=_native.DECODE_MMA) == _native.OK
    assert call(1, dtype=_native.DTYPE_F32, variant=_native.DECODE_AUTO) == _native.OK  # fp32 plans the FMA kernel


def test_plan_stream_workspace_holds_the_schedule():
    """The stream kernel's workspace: the per-warp descriptors and partial
    slots, then the per-step schedule (header, tile prefix and context
    lengths, the rows in stream order, per-warp records of 144 bytes)."""
    p = _plan(variant="stream", num_seqs=256, max_blocks_per_seq=128)
    warps = 148 * 3 * 4  # 3 CTAs of 4 warps per SM at head_dim 64 (an upper bound: the plan sizes for it)
    tiles = 256 * 2 * 128
    assert p["workspace_bytes"] >= 256 + warps * 144 + tiles * 4 + (2 * 256 + 1) * 4


def test_direct_binding_loads_and_routes_cpu_tensors_to_the_full_path():
    """The C++ binding of the per-step calls loads without a GPU and declines
    (SLOW_PATH) anything but CUDA tensors, leaving the Python wrapper's checks
    to raise the documented errors."""
    fast = _native.fast()
    assert fast.SLOW_PATH == -1000
    k = torch.zeros(2, 2, 64, dtype=torch.bfloat16)
    kc = torch.zeros(4, 2, 16, 64, dtype=torch.bfloat16)
    assert fast.kv_write(k, k, kc, kc, torch.zeros(2, dtype=torch.int64), 16, True, 0) == fast.SLOW_PATH
    q = torch.zeros(2, 4, 64, dtype=torch.bfloat16)
    st, out = fast.decode(q, kc, kc, torch.zeros(2, 1, dtype=torch.int64), torch.ones(2, dtype=torch.int32), 16,
                          -1.0, None, _native.DECODE_AUTO, 0, 0, None)
    assert st == fast.SLOW_PATH and out is None


def test_trace_build_is_separate_from_the_product_library():
    """The per-warp timeline stamps live only in the trace build
    (lib/libmvb200_trace.so, -DMVB_STREAM_TRACE); the product library the
    backend loads exports none of the trace calls."""
    from mini_vllm_b200 import build as B

    raw = ctypes.CDLL(_native.LIB_PATH)
    assert not hasattr(raw, "mvb_trace_clear") and not hasattr(raw, "mvb_trace_read")
    if not os.path.exists(B.TRACE_LIB_PATH):
        pytest.skip("trace build not made (build.build_trace())")
    trace = ctypes.CDLL(B.TRACE_LIB_PATH)
    assert hasattr(trace, "mvb_trace_clear") and hasattr(trace, "mvb_trace_read")
    assert trace.mvb_abi_version() == _native.ABI_VERSION
    for name in declared_symbols():
        assert hasattr(trace, name), name

"""The C ABI library loads, exports every declared entry point, and rejects
bad jobs on the host before touching the device (no GPU needed)."""
from __future__ import annotations

import ctypes
import re

from conftest import ROOT


def declared_symbols():
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"KB200_API\s+[\w\s\*]+?\b(kb200_\w+)\s*\(", header.read_text()))
    return sorted(names)


def test_every_declared_symbol_is_exported(kb):
    names = declared_symbols()
    assert len(names) >= 10
    for name in names:
        assert hasattr(kb.lib, name), name


def test_status_names_follow_reference_messages(kb):
    assert kb.lib.kb200_status_name(kb.NONFINITE_WEIGHT) == b"h3_cuda_nonfinite_weight"
    assert kb.lib.kb200_status_name(kb.ALIAS) == b"h3_cuda_alias"
    assert kb.lib.kb200_status_name(kb.CANCELLED) == b"h3_cuda_cancelled"


def test_block_geometry_matches_oracle(kb, oracle):
    for e in (kb.Q8_0, kb.Q4_K, kb.Q6_K, kb.Q3_K, kb.IQ4_NL, kb.IQ4_XS, kb.BF16):
        assert kb.lib.kb200_encoding_supported(e) == 1
        assert kb.block_values(e) == oracle.block_values(e)
        assert kb.block_bytes(e) == oracle.block_bytes(e)
    for e in (kb.IQ3_XXS, kb.IQ2_S, kb.IQ3_S, 42):
        assert kb.lib.kb200_encoding_supported(e) == 0


FAKE_W, FAKE_X, FAKE_Y = 0x10000000, 0x20000000, 0x30000000


def job(kb, **kw):
    base = dict(weights=FAKE_W, input=FAKE_X, output=FAKE_Y, status=None, row_bytes=2304, stride=64,
                in_=4096, columns=64, rows=1, encoding=kb.Q4_K)
    base.update(kw)
    return kb.GemvJob(**base)


def call(kb, jobs):
    arr = (kb.GemvJob * len(jobs))(*jobs)
    return kb.lib.kb200_gguf_gemv_batch(arr, len(jobs), None)


def test_unsupported_before_any_launch(kb):
    # gguf_batch_supported rules (IW/include/kadan/gguf_batch_partition.hpp:12-31).
    assert call(kb, [job(kb, encoding=kb.IQ2_S)]) == kb.UNSUPPORTED
    assert call(kb, [job(kb, in_=4100)]) == kb.UNSUPPORTED
    assert call(kb, [job(kb, rows=0)]) == kb.UNSUPPORTED
    assert call(kb, [job(kb, rows=4097)]) == kb.UNSUPPORTED
    assert call(kb, [job(kb, in_=4096 + 128)]) == kb.UNSUPPORTED  # not whole Q4_K blocks
    # one bad job rejects the whole batch
    assert call(kb, [job(kb), job(kb, encoding=99)]) == kb.UNSUPPORTED


def test_invalid_and_alias_are_reported(kb):
    assert call(kb, [job(kb, weights=None)]) == kb.INVALID
    assert call(kb, [job(kb, row_bytes=100)]) == kb.INVALID
    assert call(kb, [job(kb, stride=10)]) == kb.INVALID
    assert call(kb, [job(kb, output=FAKE_X + 64)]) == kb.ALIAS
    # output of one job over the input of another
    assert call(kb, [job(kb), job(kb, output=FAKE_X + 1024, input=0x50000000)]) == kb.ALIAS
    assert b"alias" in kb.lib.kb200_last_error()


def test_path_selection(kb):
    # 2 (tensor pipe) needs the driver's tensor-map encoder, absent without a GPU driver.
    assert kb.gemv_path(job(kb)) in (1, 2)
    assert kb.gemv_path(job(kb, encoding=kb.Q8_0, row_bytes=4352)) == 1
    assert kb.gemv_path(job(kb, weights=FAKE_W + 2)) == 0          # unaligned base
    assert kb.gemv_path(job(kb, encoding=kb.Q8_0, in_=160, row_bytes=170)) == 0
    assert kb.gemv_path(job(kb, encoding=kb.Q3_K, row_bytes=16 * 110)) == 0
    assert kb.gemv_path(job(kb, encoding=kb.F32, row_bytes=4096 * 4)) == 0
    assert kb.gemv_path(job(kb, encoding=kb.IQ2_S)) == -1


def test_dequant_rejects_partial_blocks(kb):
    assert kb.lib.kb200_gguf_dequant(kb.Q4_K, FAKE_W, 100, FAKE_Y, None, None) == kb.INVALID
    assert kb.lib.kb200_gguf_dequant(kb.IQ2_S, FAKE_W, 256, FAKE_Y, None, None) == kb.UNSUPPORTED
    assert kb.lib.kb200_gguf_dequant(kb.Q4_K, FAKE_W, 256, FAKE_W + 16, None, None) == kb.ALIAS


def test_gemv_allreduce_rejects_bad_groups_before_any_launch(kb):
    from kadan_b200 import collectives  # noqa: F401  (declares the argument types)

    peers = (ctypes.c_void_p * 2)(0x40000000, 0x48000000)

    def ar(j, world=2, rank=0, peers_=peers, max_count=1 << 20):
        return kb.lib.kb200_gguf_gemv_allreduce(None if j is None else ctypes.byref(j), peers_, world, rank,
                                                max_count, 2.0, None)

    assert ar(None) == kb.INVALID
    assert ar(job(kb, encoding=kb.IQ2_S)) == kb.UNSUPPORTED
    assert ar(job(kb), world=9) == kb.UNSUPPORTED
    assert ar(job(kb), rank=2) == kb.UNSUPPORTED
    assert ar(job(kb, stride=128)) == kb.INVALID  # output rows must be contiguous
    assert ar(job(kb), peers_=None) == kb.INVALID
    assert ar(job(kb, columns=63, stride=63)) == kb.INVALID  # odd number of values
    assert ar(job(kb, rows=4, stride=64), max_count=128) == kb.INVALID  # more values than the buffers hold


def test_peer_allreduce_host_checks(kb):
    from kadan_b200 import collectives  # noqa: F401

    assert kb.lib.kb200_peer_buffer_bytes(0, 1024) == 0
    assert kb.lib.kb200_peer_buffer_bytes(9, 1024) == 0
    assert kb.lib.kb200_peer_buffer_bytes(2, 8192) == 4096 + 2 * 8 * 8192 * 8
    peers = (ctypes.c_void_p * 2)(0x40000000, 0x48000000)
    f = kb.lib.kb200_peer_allreduce_f32
    assert f(FAKE_Y, 8192, peers, 9, 0, 8192, 2.0, None) == kb.UNSUPPORTED
    assert f(FAKE_Y, 8192, peers, 1, 0, 8192, 2.0, None) == kb.OK  # one rank: nothing to add
    assert f(FAKE_Y, 8191, peers, 2, 0, 8192, 2.0, None) == kb.INVALID
    assert f(FAKE_Y, 16384, peers, 2, 0, 8192, 2.0, None) == kb.INVALID
    assert f(FAKE_Y, 8192, None, 2, 0, 8192, 2.0, None) == kb.INVALID
    misaligned = (ctypes.c_void_p * 2)(0x40000000, 0x48000010)
    assert f(FAKE_Y, 8192, misaligned, 2, 0, 8192, 2.0, None) == kb.INVALID


def test_moe_stages_host_checks(kb):
    lib = kb.lib
    assert lib.kb200_moe_dispatch_workspace_bytes(64, 100, 32, 4) == 0  # hidden not a multiple of 64
    assert lib.kb200_moe_dispatch_workspace_bytes(64, 2880, 32, 4) > 64 * 4 * 2880 * 2
    d = kb.MoeDispatch()
    ws = 0x60000000
    assert lib.kb200_moe_dispatch_rows(FAKE_X, FAKE_Y, 64, 2880, 32, 4, ws, 1 << 30, None, None, None) == kb.INVALID
    assert lib.kb200_moe_dispatch_rows(FAKE_X, FAKE_Y, 0, 2880, 32, 4, ws, 1 << 30, ctypes.byref(d), None,
                                       None) == kb.OK
    assert d.count == 0
    assert lib.kb200_moe_dispatch_rows(FAKE_X, FAKE_Y, 64, 2880, 32, 40, ws, 1 << 30, ctypes.byref(d), None,
                                       None) == kb.UNSUPPORTED  # top_k above 32
    assert lib.kb200_moe_dispatch_rows(None, FAKE_Y, 64, 2880, 32, 4, ws, 1 << 30, ctypes.byref(d), None,
                                       None) == kb.INVALID
    assert lib.kb200_moe_dispatch_rows(FAKE_X, FAKE_Y, 64, 2880, 32, 4, ws, 1024, ctypes.byref(d), None,
                                       None) == kb.NO_MEMORY
    w = kb.MoeWeights(0x70000000, 0x71000000, None, 0x72000000, 0x73000000, None, 2880, 2880, 2, 4, 0, 1, 7.0, 1.702)
    # The expert stage ignores top_k (a rank may hold fewer experts than k).
    assert lib.kb200_moe_experts_workspace_bytes(ctypes.byref(w), 100) > 0
    assert lib.kb200_moe_experts(ctypes.byref(w), FAKE_X, FAKE_Y, 0, FAKE_Y, ws, 1 << 30, None, None) == kb.OK
    assert lib.kb200_moe_experts(ctypes.byref(w), None, FAKE_Y, 10, FAKE_Y, ws, 1 << 30, None, None) == kb.INVALID
    assert lib.kb200_moe_experts(ctypes.byref(w), FAKE_X, FAKE_Y, 10, FAKE_Y, ws, 16, None, None) == kb.NO_MEMORY
    c = lib.kb200_moe_combine
    assert c(FAKE_X, FAKE_Y, FAKE_W, 10, 0, 2880, FAKE_Y, None) == kb.UNSUPPORTED
    assert c(FAKE_X, FAKE_Y, FAKE_W, 10, 4, 2882, FAKE_Y, None) == kb.UNSUPPORTED
    assert c(FAKE_X, FAKE_Y, FAKE_W, 0, 4, 2880, FAKE_Y, None) == kb.OK
    assert c(None, FAKE_Y, FAKE_W, 10, 4, 2880, FAKE_Y, None) == kb.INVALID
    assert c(FAKE_X + 4, FAKE_Y, FAKE_W, 10, 4, 2880, FAKE_Y, None) == kb.INVALID
    r = lib.kb200_rows_regroup
    segs = 0x74000000
    assert r(FAKE_X, FAKE_Y, 5760, segs, 0, 0, None) == kb.OK
    assert r(FAKE_X, FAKE_Y, 5762, segs, 4, 10, None) == kb.INVALID
    assert r(None, FAKE_Y, 5760, segs, 4, 10, None) == kb.INVALID
    assert r(FAKE_X, FAKE_Y, 5760, segs, 70000, 10, None) == kb.UNSUPPORTED


def test_expert_exchange_host_checks(kb):
    from kadan_b200 import collectives  # noqa: F401

    lib = kb.lib
    assert lib.kb200_ep_buffer_bytes(9, 128, 2880, 1024, 256) == 0
    assert lib.kb200_ep_buffer_bytes(2, 300, 2880, 1024, 256) == 0
    assert lib.kb200_ep_buffer_bytes(2, 128, 2880, 1024, 256) > 1024 * 2880 * 2 + 256 * 2880 * 4
    assert lib.kb200_ep_rows_area(None) is None
    peers = (ctypes.c_void_p * 2)(0x40000000, 0x48000000)
    lo = 0x76000000

    def dispatch(world=2, rank=0, experts=128, hidden=2880, peers_=peers, rows=FAKE_X, offsets=FAKE_W):
        return lib.kb200_ep_dispatch(offsets, rows, hidden, experts, world, rank, peers_, 1024, 256, lo, 2.0, None)

    assert dispatch(world=9) == kb.UNSUPPORTED
    assert dispatch(rank=2) == kb.UNSUPPORTED
    assert dispatch(experts=127) == kb.UNSUPPORTED  # not an even split over 2 ranks
    assert dispatch(hidden=2890) == kb.UNSUPPORTED
    assert dispatch(peers_=None) == kb.INVALID
    assert dispatch(peers_=(ctypes.c_void_p * 2)(0x40000000, 0x48000040)) == kb.INVALID
    assert dispatch(rows=None) == kb.INVALID
    assert dispatch(rows=FAKE_X + 8) == kb.INVALID
    ret = lib.kb200_ep_return
    assert ret(None, 2880, 128, 2, 0, peers, 1024, 256, 2.0, None) == kb.INVALID
    assert ret(FAKE_Y + 4, 2880, 128, 2, 0, peers, 1024, 256, 2.0, None) == kb.INVALID
    assert ret(FAKE_Y, 2880, 128, 2, 0, peers, 0, 256, 2.0, None) == kb.INVALID


def test_new_entry_points_reject_bad_arguments_on_host(kb):
    """Bank, reader, shard and source-batch entry points refuse null handles
    and bad arguments on the host, with a status and no crash."""
    import ctypes

    from kadan_b200 import gguf_file, shard, weight_bank  # noqa: F401 - declares the prototypes

    L = kb.lib
    out = ctypes.c_void_p()
    assert L.kb200_bank_create(1024, None, ctypes.byref(out)) == kb.INVALID and not out.value
    assert L.kb200_bank_find(None, None, ctypes.byref(out)) == kb.INVALID
    assert L.kb200_bank_release(None) == kb.INVALID
    assert L.kb200_bank_bound(None, 5) == kb.INVALID
    assert L.kb200_bank_release_sources(None, None, 0, None) == kb.INVALID
    L.kb200_bank_destroy(None)
    assert L.kb200_gguf_open(None, None, ctypes.byref(out)) != kb.OK and not out.value
    assert L.kb200_gguf_open(b"/nonexistent-dir-for-kb200", None, ctypes.byref(out)) == kb.IO
    assert L.kb200_gguf_tensor_count(None) == 0
    assert L.kb200_gguf_read_packed_rows(None, b"x", 0, 0, None, 0, None) == kb.INVALID
    assert L.kb200_gguf_rows_source(None, 0, None, 0) == kb.INVALID
    L.kb200_gguf_close(None)
    assert L.kb200_shard_open(b"/nonexistent-dir-for-kb200", b"s.safetensors", None, ctypes.byref(out)) == kb.IO
    assert L.kb200_shard_open(b".", b"../escape", None, ctypes.byref(out)) == kb.INVALID
    assert L.kb200_shard_tensor_count(None) == 0
    assert L.kb200_shard_load_mxfp4_expert_rows(None, b"p", 0, 0, 1, 1, None, 0, None, 0, None) == kb.INVALID
    L.kb200_shard_close(None)
    result = ctypes.c_int(7)
    assert L.kb200_dense_gguf_source_batch(None, None, None, 0, 0, None, ctypes.byref(result)) == kb.UNSUPPORTED
    assert result.value == kb.RESULT_UNSUPPORTED
    assert L.kb200_dense_gguf_source(None, None, None, None, 0, 0, None, ctypes.byref(result)) == kb.UNSUPPORTED
    assert L.kb200_context_set_read_lanes(None, 4) == kb.INVALID
    assert L.kb200_source_job_supported(None) == 0
    assert kb.lib.kb200_status_name(kb.QUARANTINED) == b"weight_cleanup_unconfirmed"
    assert kb.lib.kb200_status_name(kb.NONFINITE_BIAS) == b"h3_cuda_nonfinite_bias"
    assert kb.lib.kb200_status_name(kb.NONFINITE_OUTPUT) == b"h3_cuda_nonfinite_output"


def test_gemm_supported_predicate(kb):
    """kb200_gguf_gemm_supported (host only): Q4_K, Q6_K and Q8_0 in whole
    256-value steps with 16-byte aligned rows of a 16-byte multiple pitch."""
    def job(enc, in_, row_bytes, ptr=0x10000):
        return kb.GemvJob(ptr, 0x200000, 0x300000, None, row_bytes, 64, in_, 64, 16, enc)

    assert kb.gemm_supported(job(kb.Q4_K, 4096, 2304))
    assert kb.gemm_supported(job(kb.Q6_K, 8192, 6720))
    assert kb.gemm_supported(job(kb.Q6_K, 4096, 3360))
    assert kb.gemm_supported(job(kb.Q8_0, 4096, 4352))
    assert not kb.gemm_supported(job(kb.Q6_K, 1024, 840))   # 840-byte rows: not a 16-byte pitch
    assert kb.gemm_supported(job(kb.Q6_K, 1024, 848))       # the same rows padded
    assert not kb.gemm_supported(job(kb.Q8_0, 4128, 4386))  # not whole 256-value steps
    assert not kb.gemm_supported(job(kb.Q4_K, 4096, 2304, ptr=0x10008))  # unaligned weights
    assert not kb.gemm_supported(job(kb.Q4_K, 4096, 2288))  # rows shorter than K
    for enc in (kb.Q3_K, kb.IQ4_NL, kb.IQ4_XS, kb.BF16, kb.F32):
        assert not kb.gemm_supported(job(enc, 4096, 8192))


def test_layer_math_host_checks(kb):
    """Shape rules of the layer-math entries are checked before any launch."""
    L = kb.lib
    fake = ctypes.c_void_p(0x10000000)
    # gguf_text_rope_shape: odd rotary, rotary above the head width, ragged rows.
    assert L.kb200_rope(fake, 1, 128, 128, 127, 0, 10000.0, None) == kb.INVALID
    assert L.kb200_rope(fake, 1, 128, 64, 128, 0, 10000.0, None) == kb.INVALID
    assert L.kb200_rope(fake, 1, 100, 64, 64, 0, 10000.0, None) == kb.INVALID
    # Attention: head dims 64/128/256, at most 16 query heads per KV head.
    assert L.kb200_attend_supported(64, 8, 128) == 1
    assert L.kb200_attend_supported(64, 8, 96) == 0
    assert L.kb200_attend_supported(64, 2, 128) == 0
    assert L.kb200_attend_supported(16, 1, 256) == 0
    assert L.kb200_attend_supported(6, 4, 128) == 0
    assert L.kb200_attend_cached(fake, fake, fake, 1, 0, 64, 2, 128, 1.0, None, None, fake, fake, 1 << 20,
                                 None) == kb.UNSUPPORTED
    need = L.kb200_attend_workspace_bytes(2, 300, 8, 64)
    assert need == 2 * 8 * 3 * 66 * 4  # at most one segment per 128 keys
    assert L.kb200_attend_cached(fake, fake, fake, 2, 300, 8, 2, 64, 1.0, None, None, ctypes.c_void_p(0x20000000),
                                 fake, need - 1, None) == kb.NO_MEMORY
    # Delta net: dim a multiple of 32 up to 256, value heads a multiple of key heads.
    assert L.kb200_delta_supported(16, 32, 128, 4) == 1
    assert L.kb200_delta_supported(16, 24, 128, 4) == 0
    assert L.kb200_delta_supported(2, 4, 96 + 8, 4) == 0
    assert L.kb200_delta_supported(2, 4, 512, 4) == 0
    args = kb.DeltaArgs(rows=1, key_heads=3, value_heads=4, dim=128, kernel=4)
    assert L.kb200_delta_step(ctypes.byref(args), fake, 1 << 20, None) == kb.UNSUPPORTED
    args = kb.DeltaArgs(rows=2, key_heads=2, value_heads=4, dim=64, kernel=4)
    assert L.kb200_delta_workspace_bytes(ctypes.byref(args)) == ((2 + 3) * (2 * 2 + 4) * 64 * 4 + 255) // 256 * 256

"""The resident weight bank (kb200_bank_*) against a host-side fake of its
device operations: the ownership rules of the reference's DeviceWeights
(services/hikari/inference_worker/include/kadan/device_weights.hpp:35-486),
scenario by scenario as the reference's own tests/device_weights.cpp checks
them — piecewise admission and late publication, refusals that touch
nothing, rollbacks, quarantine after a failed cleanup, cancellation, key
identity, stage retirement and the envelope bound. No GPU."""
from __future__ import annotations

import ctypes

import pytest

PIECE = 1024 * 1024


@pytest.fixture(scope="module")
def wb():
    from kadan_b200 import weight_bank

    return weight_bank


class Fake:
    """WeightDeviceOperations stand-in. Handles are small integers that are
    never dereferenced; every contract breach is recorded in `breaches`."""

    def __init__(self, free_bytes=1024):
        self.free_bytes = free_bytes
        self.pointers = {}
        self.events = []
        self.device_copies = []  # (offset, size, source)
        self.host_copies = 0
        self.frees = 0
        self.fail = set()
        self.oom = False
        self.synchronized = False
        self.cancel = None  # a ctypes.c_ubyte the copies set, if given
        self.on_copy = None
        self.on_sync = None
        self.breaches = []
        self._next = 0

    def available_weight_bytes(self):
        return self.free_bytes

    def allocate_weight(self, nbytes):
        self.events.append("allocate")
        if self.oom:
            return None
        if "allocate" in self.fail:
            raise RuntimeError("allocate")
        self._next += 1
        self.pointers[self._next] = nbytes
        return self._next

    def _check_copy(self, dst, offset, nbytes):
        if dst not in self.pointers or nbytes > PIECE or offset + nbytes > self.pointers[dst]:
            self.breaches.append(("copy", dst, offset, nbytes))

    def copy_weight(self, dst, offset, src, nbytes):
        self._check_copy(dst, offset, nbytes)
        self.host_copies += 1
        self.events.append("copy_host")
        if self.on_copy:
            self.on_copy()
        if self.cancel is not None:
            self.cancel.value = 1
        if "copy" in self.fail:
            raise RuntimeError("copy")

    def copy_weight_device(self, dst, offset, src, nbytes):
        self._check_copy(dst, offset, nbytes)
        self.device_copies.append((offset, nbytes, src))
        self.events.append("copy_device")
        if self.on_copy:
            self.on_copy()
        if self.cancel is not None:
            self.cancel.value = 1
        if "copy_device" in self.fail:
            raise RuntimeError("copy_device")

    def free_weight(self, p):
        if not self.synchronized:
            self.breaches.append(("free before synchronize", p))
        self.synchronized = False
        self.events.append("free")
        if "free" in self.fail:
            raise RuntimeError("free")
        if self.pointers.pop(p, None) is None:
            self.breaches.append(("unknown free", p))
        self.frees += 1

    def synchronize_weights(self):
        self.events.append("sync")
        if self.on_sync:
            self.on_sync()
        self.synchronized = True
        if "sync" in self.fail:
            raise RuntimeError("sync")


def buffer(nbytes, fill=0):
    b = (ctypes.c_ubyte * max(1, nbytes))()
    ctypes.memset(b, fill, nbytes)
    return b, ctypes.addressof(b)


def key(wb, first=0, count=8, width=4, **source):
    return wb.WeightKey(wb.WeightIdentity(**{"device": 1, **source}), first, count, width)


def raises(status, fn):
    from kadan_b200 import KadanError

    with pytest.raises(KadanError) as e:
        fn()
    assert e.value.status == status, (e.value.status, str(e.value))
    return str(e.value)


def test_device_copy_is_piecewise_and_published_last(wb):
    gpu = Fake(free_bytes=8 * PIECE)
    bank = wb.WeightBank(8 * PIECE, gpu)
    k = key(wb, first=10, count=70001, width=34, inode=7)
    scratch, addr = buffer(k.count * k.width, 0x5A)
    seen = []
    gpu.on_copy = gpu.on_sync = lambda: seen.append(bank.find(k))
    p = bank.retain_device(k, addr, k.count * k.width)
    assert p and bank.find(k) == p and gpu.host_copies == 0
    assert seen and all(s is None for s in seen)  # never visible before it is complete
    assert gpu.events == ["allocate", "copy_device", "copy_device", "copy_device", "sync"]
    assert [c[0] for c in gpu.device_copies] == [0, PIECE, 2 * PIECE]
    assert [c[1] for c in gpu.device_copies] == [PIECE, PIECE, k.count * k.width - 2 * PIECE]
    assert all(c[2] == addr for c in gpu.device_copies)
    assert bank.allocated() == k.count * k.width
    # A hit needs neither free memory nor a copy.
    gpu.on_copy = gpu.on_sync = None
    before = list(gpu.events)
    gpu.free_bytes = 0
    assert bank.retain_device(k, addr, k.count * k.width) == p
    assert gpu.events == before
    bank.release()
    assert not gpu.pointers and bank.reserved() == 0 and not gpu.breaches


def test_refusals_touch_nothing(wb):
    gpu = Fake()
    bank = wb.WeightBank(64, gpu)
    k = key(wb, count=16, width=4)
    scratch, addr = buffer(64, 0x6B)
    p = bank.retain_device(k, addr, 64)
    assert p and len(gpu.device_copies) == 1
    beyond = key(wb, first=16, count=16, width=4)
    before = list(gpu.events)
    assert bank.retain_device(beyond, addr, 64) is None
    assert bank.last_refusal == wb.ENVELOPE
    assert bank.find(beyond) is None and bank.find(k) == p
    assert gpu.events == before and bytes(scratch) == b"\x6b" * 64
    assert bank.allocated() == 64 and len(gpu.pointers) == 1
    bank.release()

    for oom in (False, True):
        gpu = Fake(free_bytes=1024 if oom else 0)
        gpu.oom = oom
        bank = wb.WeightBank(64, gpu)
        assert bank.retain_device(k, addr, 64) is None
        assert bank.last_refusal == (wb.ALLOCATION if oom else wb.PHYSICAL)
        assert not gpu.device_copies and not gpu.pointers
        assert bank.allocated() == 0 and not bank.quarantined()
        bank.release()
    gpu = Fake()
    bank = wb.WeightBank(64, gpu)
    assert bank.retain(key(wb, count=0, width=4), None, 0) is None and bank.last_refusal == wb.EMPTY


def test_failed_admission_rolls_back(wb):
    from kadan_b200 import CUDA

    k = key(wb)
    scratch, addr = buffer(32)
    for failure in ("allocate", "copy_device"):
        gpu = Fake()
        bank = wb.WeightBank(64, gpu)
        gpu.fail = {failure}
        msg = raises(CUDA, lambda: bank.retain_device(k, addr, 32))
        assert failure in msg
        assert not bank.quarantined() and bank.allocated() == 0 and not gpu.pointers
        assert bank.find(k) is None
        if failure == "copy_device":
            assert gpu.events == ["allocate", "copy_device", "sync", "free"]
        gpu.fail = set()
        bank.release()
        assert bank.reserved() == 0 and not gpu.breaches


def test_failed_rollback_quarantines(wb):
    from kadan_b200 import QUARANTINED

    k = key(wb)
    scratch, addr = buffer(32)
    for failure in ("sync", "free"):
        gpu = Fake()
        bank = wb.WeightBank(64, gpu)
        gpu.fail = {"sync"} if failure == "sync" else {"copy_device", "free"}
        msg = raises(QUARANTINED, lambda: bank.retain_device(k, addr, 32))
        operation = "synchronize" if failure == "sync" else "copy_device"
        cleanup = "synchronize" if failure == "sync" else "free"
        assert msg.index(operation) < msg.index("; cleanup:") < msg.rindex(cleanup)
        assert bank.quarantined() and bank.allocated() == 32 and len(gpu.pointers) == 1
        assert bank.reserved() == 64
        raises(QUARANTINED, lambda: bank.find(k))
        raises(QUARANTINED, lambda: bank.release())
        frees = gpu.frees
        bank.close()  # a quarantined bank's entries are not freed again
        assert gpu.frees == frees


def test_cancel_between_pieces_rolls_back(wb):
    from kadan_b200 import CANCELLED

    gpu = Fake(free_bytes=4 * PIECE)
    bank = wb.WeightBank(4 * PIECE, gpu)
    k = key(wb, count=(2 * PIECE + 32) // 4, width=4)
    scratch, addr = buffer(k.count * k.width)
    cancel = ctypes.c_ubyte(0)
    gpu.cancel = cancel
    raises(CANCELLED, lambda: bank.retain_device(k, addr, k.count * k.width, cancel))
    assert cancel.value == 1 and len(gpu.device_copies) == 1 and gpu.device_copies[0][1] == PIECE
    assert not gpu.pointers and not bank.quarantined() and bank.allocated() == 0
    # Cancellation observed after the last piece and the synchronise rolls back too.
    gpu = Fake()
    bank = wb.WeightBank(64, gpu)
    cancel = ctypes.c_ubyte(0)
    gpu.cancel = cancel
    raises(CANCELLED, lambda: bank.retain(key(wb), addr, 32, cancel))
    assert bank.allocated() == 0 and not gpu.pointers


def test_argument_checks_precede_device_work(wb):
    from kadan_b200 import CANCELLED, INVALID

    gpu = Fake()
    bank = wb.WeightBank(64, gpu)
    k = key(wb)
    scratch, addr = buffer(32)
    raises(CANCELLED, lambda: bank.retain_device(k, addr, 32, ctypes.c_ubyte(1)))
    assert "weight_device_source" in raises(INVALID, lambda: bank.retain_device(k, None, 32))
    assert "weight_representation_size" in raises(INVALID, lambda: bank.retain_device(k, addr, 31))
    huge = key(wb, count=2**63, width=144)
    raises(INVALID, lambda: bank.retain(huge, addr, 32))
    raises(INVALID, lambda: bank.retain(key(wb, count=8, width=0), addr, 0))
    assert gpu.events == [] and bank.reserved() == 0


def test_keys_separate_widths_sources_and_rows(wb):
    from kadan_b200 import CANCELLED, INVALID

    gpu = Fake(free_bytes=2048)
    bank = wb.WeightBank(1024, gpu)
    packed, addr = buffer(288)
    reads = []

    def fetch(k):
        hit = bank.find(k)
        if hit:
            return hit
        reads.append(k)
        return bank.retain(k, addr, k.count * k.width)

    got = []
    for width in (110, 144, 34, 4):  # Q3_K, Q4_K, Q8_0 and F32 tiles over one block range
        k = key(wb, count=2, width=width)
        assert bank.find(k) is None
        got.append(fetch(k))
        assert got[-1] and got[-1] not in got[:-1]
        assert fetch(k) == got[-1]
    assert len(reads) == 4 and gpu.host_copies == 4 and bank.allocated() == 584
    expert = key(wb, count=2, width=110, payload_begin=220, payload_end=440)
    assert bank.find(expert) is None and fetch(expert)
    assert bank.allocated() == 804
    next_rows = key(wb, first=2, count=2, width=110, payload_begin=220, payload_end=440)
    assert fetch(next_rows) and bank.allocated() == 1024
    assert fetch(key(wb, first=4, count=2, width=110, payload_begin=220, payload_end=440)) is None
    assert gpu.host_copies == 6 and bank.allocated() == 1024
    # Retirement is not cancellable and drops exactly that tensor's tiles.
    assert bank.release_sources([expert.source]) == 440
    raises(CANCELLED, lambda: bank.retain(key(wb, count=2, width=4), addr, 8, ctypes.c_ubyte(1)))
    assert bank.find(key(wb, count=2, width=4)) == got[-1]
    raises(INVALID, lambda: bank.retain(key(wb, count=2, width=110), addr, 219))
    assert bank.allocated() == 584 and gpu.host_copies == 6
    bank.release()
    assert gpu.frees == 6 and not gpu.pointers and not gpu.breaches


def test_stage_retirement_makes_room(wb):
    capacity = 2 * (110 + 144 + 34)
    gpu = Fake()
    bank = wb.WeightBank(capacity, gpu)
    packed, addr = buffer(288)
    widths = (110, 144, 34)
    prefill = [key(wb, first=2, count=2, width=w, inode=77, payload_begin=i * 4096, payload_end=(i + 1) * 4096)
               for i, w in enumerate(widths)]
    for k in prefill:
        assert bank.retain(k, addr, k.count * k.width)
    assert bank.allocated() == capacity and gpu.host_copies == 3
    later = key(wb, first=2, count=2, width=110, inode=77, payload_begin=12288, payload_end=16384)
    assert bank.retain(later, addr, 220) is None and bank.last_refusal == wb.ENVELOPE
    unrelated = bank.find(prefill[2])
    assert bank.release_sources([prefill[0].source, prefill[1].source]) == 2 * (110 + 144)
    assert bank.find(prefill[0]) is None and bank.find(prefill[1]) is None
    assert bank.find(prefill[2]) == unrelated and bank.allocated() == 68
    assert bank.release_sources([prefill[2].source]) == 68
    assert bank.allocated() == 0 and not gpu.pointers
    # The envelope stays charged across a retirement.
    assert bank.reserved() == capacity and bank.capacity() == capacity == bank.maximum_capacity()
    decode = [key(wb, first=4 + 2 * i, count=2, width=w, inode=77, payload_begin=12288 + i * 4096,
                  payload_end=12288 + (i + 1) * 4096) for i, w in enumerate(widths)]
    ptrs = [bank.retain(k, addr, k.count * k.width) for k in decode]
    assert all(ptrs) and bank.allocated() == capacity and gpu.host_copies == 6
    assert [bank.retain(k, addr, k.count * k.width) for k in decode] == ptrs
    assert gpu.host_copies == 6 and gpu.frees == 3
    bank.release()
    assert gpu.frees == 6 and bank.reserved() == 0


def test_bound_only_before_admission(wb):
    from kadan_b200 import INVALID

    gpu = Fake()
    bank = wb.WeightBank(64, gpu)
    k = key(wb)
    vals, addr = buffer(32)
    first = bank.retain(k, addr, 32)
    assert first and bank.allocated() == 32 and bank.reserved() == 64
    assert bank.retain(k, addr, 32) == first and gpu.host_copies == 1
    assert bank.retain(key(wb, first=8), addr, 32)
    assert bank.retain(key(wb, first=16), addr, 32) is None and bank.allocated() == 64
    assert "weight_plan_already_loaded" in raises(INVALID, lambda: bank.bound(16))
    bank.release()
    assert gpu.frees == 2 and bank.reserved() == 0
    bank.bound(16)
    assert bank.capacity() == 16
    assert bank.retain(k, addr, 32) is None and bank.reserved() == 0
    bank.bound(1 << 40)  # never above the creation envelope
    assert bank.capacity() == 64
    assert bank.retain(k, addr, 32) and bank.reserved() == 64
    bank.release()


def test_physical_and_allocation_refusals_then_hit(wb):
    gpu = Fake(free_bytes=16)
    bank = wb.WeightBank(64, gpu)
    k = key(wb)
    vals, addr = buffer(32)
    assert bank.retain(k, addr, 32) is None and bank.last_refusal == wb.PHYSICAL
    assert not gpu.pointers and bank.reserved() == 0
    gpu.free_bytes, gpu.oom = 1024, True
    assert bank.retain(k, addr, 32) is None and bank.last_refusal == wb.ALLOCATION
    assert bank.allocated() == 0 and not bank.quarantined()
    gpu.oom = False
    p = bank.retain(k, addr, 32)
    assert p
    gpu.free_bytes = 0
    assert bank.retain(k, addr, 32) == p and gpu.host_copies == 1
    bank.release()


def test_release_failures_quarantine(wb):
    from kadan_b200 import CUDA, QUARANTINED

    vals, addr = buffer(32)
    k = key(wb)
    for failure in ("sync", "free"):
        for how in ("sources", "all"):
            gpu = Fake()
            bank = wb.WeightBank(64, gpu)
            assert bank.retain(k, addr, 32)
            gpu.fail = {failure}
            if how == "sources":
                raises(CUDA, lambda: bank.release_sources([k.source]))
            else:
                raises(CUDA, lambda: bank.release())
            assert bank.quarantined() and bank.allocated() == 32 and bank.reserved() == 64
            assert gpu.pointers
            gpu.fail = set()
            raises(QUARANTINED, lambda: bank.find(k))
            raises(QUARANTINED, lambda: bank.retain(k, addr, 32))
            raises(QUARANTINED, lambda: bank.release())
            raises(QUARANTINED, lambda: bank.bound(8))


def test_identity_includes_every_field(wb):
    gpu = Fake(free_bytes=1 << 20)
    bank = wb.WeightBank(1 << 20, gpu)
    vals, addr = buffer(32)
    base = dict(device=1, inode=2, file_size=3, modified_seconds=4, modified_nanoseconds=5, changed_seconds=6,
                changed_nanoseconds=7, payload_begin=8, payload_end=9)
    first = bank.retain(wb.WeightKey(wb.WeightIdentity(**base), 0, 8, 4), addr, 32)
    seen = {first}
    for name in base:
        other = dict(base, **{name: base[name] + 100})
        p = bank.retain(wb.WeightKey(wb.WeightIdentity(**other), 0, 8, 4), addr, 32)
        assert p and p not in seen
        seen.add(p)
    assert bank.entries() == 1 + len(base)
    released = bank.release_sources([wb.WeightIdentity(**base)])
    assert released == 32 and bank.entries() == len(base)
    bank.release()


def test_source_batch_checks_precede_reads(wb):
    """kb200_dense_gguf_source_batch reports an unusable call before any
    source is read (the reference's unsupported-first rule)."""
    import numpy as np

    from kadan_b200 import Q8_0, Unsupported

    calls = []

    class NoContext:
        handle = None

    job = wb.SourceJob(wb.WeightIdentity(inode=1), lambda first, n: calls.append(first) or bytes(n),
                       np.zeros((1, 64), np.float32), np.zeros((1, 8), np.float32), 64, 8, Q8_0)
    with pytest.raises(Unsupported):
        wb.dense_gguf_source_batch(NoContext(), None, [job])
    assert not calls


def test_single_source_checks_precede_reads(wb):
    """kb200_dense_gguf_source: unsupported jobs and `precise` calls return
    unsupported before any source read."""
    import numpy as np

    from kadan_b200 import Q8_0, Unsupported

    calls = []

    class NoContext:
        handle = None

    job = wb.SourceJob(wb.WeightIdentity(inode=1), lambda first, n: calls.append(first) or bytes(n),
                       np.zeros((1, 64), np.float32), np.zeros((1, 8), np.float32), 64, 8, Q8_0)
    for precise in (False, True):
        with pytest.raises(Unsupported):
            wb.dense_gguf_source(NoContext(), None, job, bias=np.zeros(8, np.float32), precise=precise)
    assert not calls

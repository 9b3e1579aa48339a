// Resident weight bank: the reference's kadan::DeviceWeights
// (services/hikari/inference_worker/include/kadan/device_weights.hpp:35-486)
// behind the C ABI. Device work goes through a table of operations so the
// bookkeeping runs the same over CUDA memory and over a host-side fake.
//
// Rules kept from the reference (each cited where it is enforced): an entry
// is published only after every piece of its copy landed and the device was
// synchronised; a failed admission is rolled back; a rollback, release or
// retirement whose synchronise or free fails quarantines the bank, and a
// quarantined bank refuses every later operation.
#include <cinttypes>
#include <cstdio>
#include <cstring>
#include <limits>
#include <map>
#include <new>
#include <string>
#include <tuple>

#include "kb200_host.hpp"

namespace kb200 {

struct CudaOps;

namespace {

constexpr uint64_t kCopyPiece = 1024 * 1024;  // device_weights.hpp:235

struct KeyLess {
    static auto tie(const kb200_weight_key& k) {
        const auto& s = k.source;
        return std::make_tuple(s.device, s.inode, s.file_size, s.modified_seconds, s.modified_nanoseconds,
                               s.changed_seconds, s.changed_nanoseconds, s.payload_begin, s.payload_end, k.first,
                               k.count, k.width);
    }
    bool operator()(const kb200_weight_key& a, const kb200_weight_key& b) const {
        return tie(a) < tie(b);
    }
};

bool same_source(const kb200_weight_identity& a, const kb200_weight_identity& b) {
    return a.device == b.device && a.inode == b.inode && a.file_size == b.file_size
           && a.modified_seconds == b.modified_seconds && a.modified_nanoseconds == b.modified_nanoseconds
           && a.changed_seconds == b.changed_seconds && a.changed_nanoseconds == b.changed_nanoseconds
           && a.payload_begin == b.payload_begin && a.payload_end == b.payload_end;
}

struct Entry {
    void* pointer = nullptr;
    uint64_t bytes = 0;
    bool ready = false;
};

// An operation's failure: its status and a description for kb200_last_error.
struct Failure {
    int status = KB200_OK;
    std::string what;
    explicit operator bool() const {
        return status != KB200_OK;
    }
};

Failure op_failure(int status, const char* op) {
    if (status == KB200_OK)
        return {};
    char text[160];
    std::snprintf(text, sizeof(text), "weight_%s failed (%s)", op, kb200_status_name(status));
    return {status, text};
}

}  // namespace
}  // namespace kb200

struct kb200_bank {
    kb200_weight_ops ops{};
    uint64_t limit = 0, maximum = 0, allocated = 0;
    bool reserved = false, quarantined = false;
    std::map<kb200_weight_key, kb200::Entry, kb200::KeyLess> entries;
    // Set when the bank owns CUDA operations (kb200_bank_create_cuda).
    kb200::CudaOps* cuda = nullptr;
};

namespace kb200 {
namespace {

int report(const Failure& f) {
    return fail(f.status, f.what.c_str());
}

bool stopped(const volatile uint8_t* cancel) {
    return cancel && *cancel;
}

// DeviceWeights::drop (device_weights.hpp:289-301): synchronise, free, then
// forget. On failure the entry stays where it is.
Failure drop(kb200_bank* b, decltype(b->entries)::iterator entry) {
    if (entry->second.pointer) {
        if (Failure f = op_failure(b->ops.synchronize(b->ops.user), "synchronize"))
            return f;
        if (Failure f = op_failure(b->ops.release(b->ops.user, entry->second.pointer), "free"))
            return f;
        b->allocated -= entry->second.bytes;
    }
    b->entries.erase(entry);
    return {};
}

// A failed admission (device_weights.hpp:256-268): roll the entry back and
// report the operation's failure; if the rollback fails too, quarantine and
// report both.
int rollback(kb200_bank* b, decltype(b->entries)::iterator entry, const Failure& cause) {
    if (Failure cleanup = drop(b, entry)) {
        b->quarantined = true;
        const std::string both = cause.what + "; cleanup: " + cleanup.what;
        return fail(KB200_QUARANTINED, both.c_str());
    }
    return report(cause);
}

int healthy(const kb200_bank* b) {
    return b->quarantined ? fail(KB200_QUARANTINED, "weight bank cleanup was not confirmed") : KB200_OK;
}

// DeviceWeights::retain_bytes (device_weights.hpp:181-270).
int retain_bytes(kb200_bank* b, const kb200_weight_key* key, const void* src, uint64_t bytes, bool device_source,
                 const volatile uint8_t* cancel, void** ptr, int* refusal) {
    if (!ptr)
        return fail(KB200_INVALID, "null output");
    *ptr = nullptr;
    if (refusal)
        *refusal = KB200_BANK_ADMITTED;
    if (!b || !key)
        return fail(KB200_INVALID, "null bank or key");
    if (bytes && !src)
        return fail(KB200_INVALID, device_source ? "weight_device_source" : "weight_host_source");
    if (const int s = healthy(b))
        return s;
    if (stopped(cancel))
        return fail(KB200_CANCELLED, "weight_cancelled");
    if (!key->width || key->count > std::numeric_limits<uint64_t>::max() / key->width
        || key->count * key->width != bytes)
        return fail(KB200_INVALID, "weight_representation_size");
    if (const auto hit = b->entries.find(*key); hit != b->entries.end() && hit->second.ready) {
        *ptr = hit->second.pointer;
        return KB200_OK;
    }
    auto refuse = [&](int why) {
        if (refusal)
            *refusal = why;
        return KB200_OK;
    };
    if (!bytes)
        return refuse(KB200_BANK_EMPTY);
    if (bytes > (b->limit > b->allocated ? b->limit - b->allocated : 0))
        return refuse(KB200_BANK_ENVELOPE);
    uint64_t available = 0;
    if (Failure f = op_failure(b->ops.available(b->ops.user, &available), "available"))
        return report(f);
    if (bytes > available)
        return refuse(KB200_BANK_PHYSICAL);
    b->reserved = true;
    auto entry = b->entries.end();
    try {
        entry = b->entries.try_emplace(*key).first;
    } catch (const std::bad_alloc&) {
        return fail(KB200_NO_MEMORY, "weight bank metadata");
    }
    void* pointer = nullptr;
    if (Failure f = op_failure(b->ops.allocate(b->ops.user, bytes, &pointer), "allocate"))
        return rollback(b, entry, f);
    if (!pointer) {
        b->entries.erase(entry);
        return refuse(KB200_BANK_ALLOCATION);
    }
    entry->second.pointer = pointer;
    entry->second.bytes = bytes;
    b->allocated += bytes;
    for (uint64_t at = 0; at < bytes; at += kCopyPiece) {
        if (stopped(cancel))
            return rollback(b, entry, {KB200_CANCELLED, "weight_cancelled"});
        const uint64_t piece = bytes - at < kCopyPiece ? bytes - at : kCopyPiece;
        const int s = device_source ? b->ops.copy_device(b->ops.user, pointer, at, src, piece)
                                    : b->ops.copy_host(b->ops.user, pointer, at, src, piece);
        if (Failure f = op_failure(s, device_source ? "copy_device" : "copy_host"))
            return rollback(b, entry, f);
    }
    if (Failure f = op_failure(b->ops.synchronize(b->ops.user), "synchronize"))
        return rollback(b, entry, f);
    if (stopped(cancel))
        return rollback(b, entry, {KB200_CANCELLED, "weight_cancelled"});
    entry->second.ready = true;
    *ptr = pointer;
    return KB200_OK;
}

bool ops_complete(const kb200_weight_ops& o) {
    return o.available && o.allocate && o.copy_host && o.copy_device && o.release && o.synchronize;
}

}  // namespace
}  // namespace kb200

namespace kb200 {

// WeightDeviceOperations over CUDA memory of one device, with a stream of the
// bank's own so its copies never wait behind projection work.
struct CudaOps {
    int device = 0;
    uint64_t scratch = 0;
    cudaStream_t stream = nullptr;
};

namespace {

int cuda_available(void* user, uint64_t* bytes) {
    auto* c = static_cast<CudaOps*>(user);
    DeviceScope scope(c->device);
    size_t free = 0, total = 0;
    const cudaError_t e = cudaMemGetInfo(&free, &total);
    if (e != cudaSuccess)
        return cuda_fail(e, "cudaMemGetInfo");
    *bytes = free > c->scratch ? free - c->scratch : 0;
    return KB200_OK;
}

int cuda_allocate(void* user, uint64_t bytes, void** out) {
    auto* c = static_cast<CudaOps*>(user);
    DeviceScope scope(c->device);
    *out = nullptr;
    const cudaError_t e = cudaMalloc(out, bytes);
    if (e == cudaErrorMemoryAllocation) {
        cudaGetLastError();  // a confirmed refusal leaves no sticky error
        *out = nullptr;
        return KB200_OK;
    }
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "cudaMalloc (weight bank)");
}

int cuda_copy(CudaOps* c, void* dst, uint64_t offset, const void* src, uint64_t bytes, cudaMemcpyKind kind) {
    DeviceScope scope(c->device);
    const cudaError_t e = cudaMemcpyAsync(static_cast<uint8_t*>(dst) + offset,
                                          static_cast<const uint8_t*>(src) + offset, bytes, kind, c->stream);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "weight bank copy");
}

int cuda_copy_host(void* user, void* dst, uint64_t offset, const void* src, uint64_t bytes) {
    return cuda_copy(static_cast<CudaOps*>(user), dst, offset, src, bytes, cudaMemcpyHostToDevice);
}

int cuda_copy_device(void* user, void* dst, uint64_t offset, const void* src, uint64_t bytes) {
    return cuda_copy(static_cast<CudaOps*>(user), dst, offset, src, bytes, cudaMemcpyDeviceToDevice);
}

int cuda_release(void* user, void* ptr) {
    auto* c = static_cast<CudaOps*>(user);
    DeviceScope scope(c->device);
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "cudaFree (weight bank)");
}

int cuda_synchronize(void* user) {
    auto* c = static_cast<CudaOps*>(user);
    DeviceScope scope(c->device);
    const cudaError_t e = cudaStreamSynchronize(c->stream);
    return e == cudaSuccess ? KB200_OK : cuda_fail(e, "weight bank synchronize");
}

}  // namespace
}  // namespace kb200

namespace kb200 {

int bank_device(const kb200_bank* bank) {
    return bank && bank->cuda ? bank->cuda->device : -1;
}

}  // namespace kb200

using namespace kb200;

extern "C" {

int kb200_bank_create(uint64_t limit, const kb200_weight_ops* ops, kb200_bank** out) {
    if (!out)
        return fail(KB200_INVALID, "null output");
    *out = nullptr;
    if (!ops || !ops_complete(*ops))
        return fail(KB200_INVALID, "weight bank operations incomplete");
    auto* b = new (std::nothrow) kb200_bank;
    if (!b)
        return fail(KB200_NO_MEMORY, "weight bank");
    b->ops = *ops;
    b->limit = b->maximum = limit;
    *out = b;
    return KB200_OK;
}

int kb200_bank_create_cuda(int device, uint64_t limit, uint64_t scratch, kb200_bank** out) {
    if (!out)
        return fail(KB200_INVALID, "null output");
    *out = nullptr;
    auto* c = new (std::nothrow) CudaOps;
    if (!c)
        return fail(KB200_NO_MEMORY, "weight bank");
    c->device = device;
    c->scratch = scratch;
    {
        DeviceScope scope(device);
        const cudaError_t e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
        if (e != cudaSuccess) {
            delete c;
            return cuda_fail(e, "cudaStreamCreate (weight bank)");
        }
    }
    const kb200_weight_ops ops{c, cuda_available, cuda_allocate, cuda_copy_host,
                               cuda_copy_device, cuda_release, cuda_synchronize};
    if (const int s = kb200_bank_create(limit, &ops, out)) {
        DeviceScope scope(device);
        cudaStreamDestroy(c->stream);
        delete c;
        return s;
    }
    (*out)->cuda = c;
    return KB200_OK;
}

void kb200_bank_destroy(kb200_bank* b) {
    if (!b)
        return;
    // A quarantined bank's entries are in an unconfirmed state: they are left
    // to the process rather than freed a second time.
    if (!b->quarantined)
        kb200_bank_release(b);
    if (b->cuda) {
        DeviceScope scope(b->cuda->device);
        cudaStreamDestroy(b->cuda->stream);
        delete b->cuda;
    }
    delete b;
}

int kb200_bank_state_get(const kb200_bank* b, kb200_bank_state* state) {
    if (!b || !state)
        return fail(KB200_INVALID, "null bank or state");
    state->capacity = b->limit;
    state->maximum_capacity = b->maximum;
    state->allocated = b->allocated;
    state->reserved = b->reserved ? b->limit : 0;
    state->entries = b->entries.size();
    state->quarantined = b->quarantined ? 1 : 0;
    return KB200_OK;
}

int kb200_bank_find(kb200_bank* b, const kb200_weight_key* key, void** ptr) {
    if (!ptr)
        return fail(KB200_INVALID, "null output");
    *ptr = nullptr;
    if (!b || !key)
        return fail(KB200_INVALID, "null bank or key");
    if (const int s = healthy(b))
        return s;
    const auto it = b->entries.find(*key);
    if (it != b->entries.end() && it->second.ready)
        *ptr = it->second.pointer;
    return KB200_OK;
}

int kb200_bank_retain(kb200_bank* b, const kb200_weight_key* key, const void* src, uint64_t bytes,
                      const volatile uint8_t* cancel, void** ptr, int* refusal) {
    return retain_bytes(b, key, src, bytes, false, cancel, ptr, refusal);
}

int kb200_bank_retain_device(kb200_bank* b, const kb200_weight_key* key, const void* src, uint64_t bytes,
                             const volatile uint8_t* cancel, void** ptr, int* refusal) {
    return retain_bytes(b, key, src, bytes, true, cancel, ptr, refusal);
}

// DeviceWeights::release_sources (device_weights.hpp:132-154).
int kb200_bank_release_sources(kb200_bank* b, const kb200_weight_identity* sources, size_t count,
                               uint64_t* released) {
    if (released)
        *released = 0;
    if (!b || (count && !sources))
        return fail(KB200_INVALID, "null bank or sources");
    if (const int s = healthy(b))
        return s;
    const uint64_t before = b->allocated;
    for (auto it = b->entries.begin(); it != b->entries.end();) {
        auto entry = it++;
        bool match = false;
        for (size_t i = 0; i < count && !match; ++i)
            match = same_source(entry->first.source, sources[i]);
        if (!match)
            continue;
        if (Failure f = drop(b, entry)) {
            b->quarantined = true;
            return report(f);
        }
    }
    if (released)
        *released = before - b->allocated;
    return KB200_OK;
}

// DeviceWeights::release (device_weights.hpp:156-179).
int kb200_bank_release(kb200_bank* b) {
    if (!b)
        return fail(KB200_INVALID, "null bank");
    if (const int s = healthy(b))
        return s;
    if (!b->entries.empty())
        if (Failure f = op_failure(b->ops.synchronize(b->ops.user), "synchronize")) {
            b->quarantined = true;
            return report(f);
        }
    while (!b->entries.empty())
        if (Failure f = drop(b, b->entries.begin())) {
            b->quarantined = true;
            return report(f);
        }
    b->reserved = false;
    return KB200_OK;
}

// DeviceWeights::bound (device_weights.hpp:75-82).
int kb200_bank_bound(kb200_bank* b, uint64_t bytes) {
    if (!b)
        return fail(KB200_INVALID, "null bank");
    if (const int s = healthy(b))
        return s;
    if (b->reserved)
        return fail(KB200_INVALID, "weight_plan_already_loaded");
    b->limit = bytes < b->maximum ? bytes : b->maximum;
    return KB200_OK;
}

}  // extern "C"

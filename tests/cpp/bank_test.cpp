// The resident weight bank (kadan_b200/csrc/weight_bank.cpp) over fake device
// operations, for runs under AddressSanitizer and UndefinedBehaviorSanitizer:
// piecewise admission, hits, refusals, a rolled-back admission, quarantine
// after a failed cleanup, retirement by identity, bound, and destruction with
// entries left. Prints "ok".
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "kadan_b200.h"
#include "kb200_host.hpp"

namespace kb200 {
int fail(int status, const char*) {
    return status;
}
int cuda_fail(cudaError_t, const char*) {
    return KB200_CUDA;
}
}  // namespace kb200

extern "C" const char* kb200_status_name(int) {
    return "status";
}

#define CHECK(c)                                                                   \
    do {                                                                           \
        if (!(c)) {                                                                \
            std::fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #c); \
            std::exit(1);                                                          \
        }                                                                          \
    } while (0)

namespace {

// Device memory played by host allocations, so copies can be checked byte for byte.
struct Fake {
    uint64_t free_bytes = 1 << 30;
    std::map<void*, std::vector<uint8_t>> blocks;
    std::string fail;  // "allocate", "copy", "sync", "free"
    bool oom = false;
    int syncs = 0, frees = 0;
};

int available(void* u, uint64_t* bytes) {
    *bytes = static_cast<Fake*>(u)->free_bytes;
    return KB200_OK;
}
int allocate(void* u, uint64_t bytes, void** out) {
    auto* f = static_cast<Fake*>(u);
    *out = nullptr;
    if (f->fail == "allocate")
        return KB200_CUDA;
    if (f->oom)
        return KB200_OK;
    std::vector<uint8_t> block(bytes);
    void* key = block.data();
    f->blocks.emplace(key, std::move(block));
    *out = key;
    return KB200_OK;
}
int copy(void* u, void* dst, uint64_t offset, const void* src, uint64_t bytes) {
    auto* f = static_cast<Fake*>(u);
    if (f->fail == "copy")
        return KB200_CUDA;
    auto& block = f->blocks.at(dst);
    CHECK(offset + bytes <= block.size() && bytes <= (1u << 20));
    std::memcpy(block.data() + offset, static_cast<const uint8_t*>(src) + offset, bytes);
    return KB200_OK;
}
int release(void* u, void* p) {
    auto* f = static_cast<Fake*>(u);
    if (f->fail == "free")
        return KB200_CUDA;
    CHECK(f->blocks.erase(p) == 1);
    ++f->frees;
    return KB200_OK;
}
int synchronize(void* u) {
    auto* f = static_cast<Fake*>(u);
    ++f->syncs;
    return f->fail == "sync" ? KB200_CUDA : KB200_OK;
}

kb200_weight_key key(uint64_t inode, uint64_t first, uint64_t count, uint64_t width) {
    kb200_weight_key k{};
    k.source.device = 1;
    k.source.inode = inode;
    k.first = first, k.count = count, k.width = width;
    return k;
}

kb200_bank* make(Fake& f, uint64_t limit) {
    const kb200_weight_ops ops{&f, available, allocate, copy, copy, release, synchronize};
    kb200_bank* b = nullptr;
    CHECK(kb200_bank_create(limit, &ops, &b) == KB200_OK);
    return b;
}

}  // namespace

int main() {
    std::vector<uint8_t> src(3 * (1u << 20) + 123);
    for (size_t i = 0; i < src.size(); ++i)
        src[i] = uint8_t(i * 7 + 3);
    {
        Fake f;
        kb200_bank* b = make(f, 8u << 20);
        const auto k = key(1, 0, src.size(), 1);
        void* p = nullptr;
        int why = -1;
        CHECK(kb200_bank_retain(b, &k, src.data(), src.size(), nullptr, &p, &why) == KB200_OK && p);
        CHECK(std::memcmp(f.blocks.at(p).data(), src.data(), src.size()) == 0);
        void* hit = nullptr;
        CHECK(kb200_bank_find(b, &k, &hit) == KB200_OK && hit == p);
        const auto big = key(2, 0, 6u << 20, 1);
        std::vector<uint8_t> large(6u << 20);
        CHECK(kb200_bank_retain(b, &big, large.data(), large.size(), nullptr, &p, &why) == KB200_OK && !p
              && why == KB200_BANK_ENVELOPE);
        const auto small = key(3, 0, 100, 1);
        CHECK(kb200_bank_retain(b, &small, src.data(), 100, nullptr, &p, &why) == KB200_OK && p);
        uint64_t released = 0;
        const kb200_weight_identity ids[] = {k.source};
        CHECK(kb200_bank_release_sources(b, ids, 1, &released) == KB200_OK && released == src.size());
        CHECK(kb200_bank_bound(b, 16) != KB200_OK);
        CHECK(kb200_bank_release(b) == KB200_OK && f.blocks.empty());
        CHECK(kb200_bank_bound(b, 16) == KB200_OK);
        CHECK(kb200_bank_retain(b, &small, src.data(), 100, nullptr, &p, &why) == KB200_OK && !p);
        // Destroyed with an entry left: it is released.
        CHECK(kb200_bank_bound(b, 1u << 20) == KB200_OK);
        CHECK(kb200_bank_retain(b, &small, src.data(), 100, nullptr, &p, &why) == KB200_OK && p);
        kb200_bank_destroy(b);
        CHECK(f.blocks.empty());
    }
    for (const char* failure : {"allocate", "copy"}) {
        Fake f;
        kb200_bank* b = make(f, 8u << 20);
        f.fail = failure;
        const auto k = key(1, 0, src.size(), 1);
        void* p = nullptr;
        CHECK(kb200_bank_retain_device(b, &k, src.data(), src.size(), nullptr, &p, nullptr) == KB200_CUDA);
        kb200_bank_state st{};
        CHECK(kb200_bank_state_get(b, &st) == KB200_OK && !st.quarantined && st.allocated == 0 && f.blocks.empty());
        kb200_bank_destroy(b);
    }
    {
        // A failed copy whose rollback cannot free: quarantined; destroy leaves the entry.
        Fake f;
        kb200_bank* b = make(f, 8u << 20);
        const auto k = key(1, 0, 64, 1);
        void* p = nullptr;
        f.fail = "copy";
        CHECK(kb200_bank_retain(b, &k, src.data(), 64, nullptr, &p, nullptr) == KB200_CUDA);
        f.fail = "sync";
        CHECK(kb200_bank_retain(b, &k, src.data(), 64, nullptr, &p, nullptr) == KB200_QUARANTINED);
        CHECK(kb200_bank_find(b, &k, &p) == KB200_QUARANTINED);
        CHECK(kb200_bank_release(b) == KB200_QUARANTINED);
        kb200_bank_destroy(b);
        CHECK(f.blocks.size() == 1);
    }
    {
        // Cancellation between pieces rolls back.
        Fake f;
        kb200_bank* b = make(f, 8u << 20);
        const auto k = key(1, 0, src.size(), 1);
        volatile uint8_t cancel = 1;
        void* p = nullptr;
        CHECK(kb200_bank_retain(b, &k, src.data(), src.size(), &cancel, &p, nullptr) == KB200_CANCELLED);
        kb200_bank_destroy(b);
        CHECK(f.blocks.empty());
    }
    std::printf("ok\n");
    return 0;
}

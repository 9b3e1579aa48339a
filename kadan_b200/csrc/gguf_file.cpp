// GGUF checkpoint reader: the reference worker's kadan::checkpoint::GgufCheckpoint
// (services/hikari/inference_worker/src/weights/gguf_checkpoint.cpp:441-674)
// over its own GGUF v3 parser (the format published with ggml: magic "GGUF",
// version, tensor and key-value counts, typed key-value pairs, tensor
// descriptors, then the aligned data section; all integers little-endian).
//
// It accepts exactly the files the reference accepts: the reference validates
// every header field itself before handing the file to ggml's parser, and
// ggml adds a few rules of its own (non-empty keys, tensor names under 64
// bytes, tensors laid out back to back at the alignment), which the reference
// reports as "gguf_invalid_metadata". The messages of failures are the
// reference's, so a caller's handling carries over.
#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <dirent.h>
#include <fcntl.h>
#include <limits>
#include <map>
#include <new>
#include <string>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>

#include "gguf_geometry.hpp"
#include "kb200_host.hpp"

namespace kb200 {
namespace {

constexpr uint64_t kMetadataLimit = 32ull << 20;       // per file (gguf_checkpoint.cpp:25)
constexpr uint64_t kSplitMetadataLimit = 64ull << 20;  // over a split set
constexpr uint64_t kMaxTensors = 200000, kMaxKeys = 16384, kMaxArray = 524288;
constexpr uint64_t kReadPiece = 1ull << 20;
constexpr size_t kMaxName = 64;                        // ggml's GGML_MAX_NAME

// GGUF value types.
enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
    kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12
};

// A failure inside the reader: the status and the reference's message.
struct Failure {
    int status;
    const char* what;
};

[[noreturn]] void raise(const char* what, int status = KB200_INVALID) {
    throw Failure{status, what};
}

void require(bool ok, const char* what) {
    if (!ok)
        raise(what);
}

uint64_t add(uint64_t a, uint64_t b) {
    require(b <= UINT64_MAX - a, "gguf_size_overflow");
    return a + b;
}

uint64_t mul(uint64_t a, uint64_t b) {
    require(!b || a <= UINT64_MAX / b, "gguf_size_overflow");
    return a * b;
}

void stop(const volatile uint8_t* cancel) {
    if (cancel && *cancel)
        raise("gguf_cancelled", KB200_CANCELLED);
}

// ggml type id -> kb200 encoding (F32 included); -2 for types the reader
// refuses. GGUF MXFP4 (ggml type 39) is refused as the reference's reader
// refuses it (gguf::encoding has no MXFP4, gguf_checkpoint.cpp:229-230) unless
// the caller opened with KB200_GGUF_ACCEPT_MXFP4; it then reads as
// KB200_GGUF_MXFP4 (32 values in 17 bytes, converted for the MoE layer by
// kb200_mxfp4_from_ggml).
int encoding_of(uint32_t ggml_type, uint32_t flags) {
    if (ggml_type == 39)
        return (flags & KB200_GGUF_ACCEPT_MXFP4) ? KB200_GGUF_MXFP4 : -2;
    switch (ggml_type) {
    case 0: return KB200_F32;
    case 8: return KB200_Q8_0;
    case 11: return KB200_Q3_K;
    case 12: return KB200_Q4_K;
    case 14: return KB200_Q6_K;
    case 18: return KB200_IQ3_XXS;
    case 20: return KB200_IQ4_NL;
    case 21: return KB200_IQ3_S;
    case 22: return KB200_IQ2_S;
    case 23: return KB200_IQ4_XS;
    case 30: return KB200_BF16;
    default: return -2;
    }
}

// An open file with the stat taken when it was opened.
struct File {
    int fd = -1;
    struct stat initial {};

    File() = default;
    File(int descriptor, bool directory) : fd(descriptor) {
        if (fd < 0)
            raise("gguf_open_failed", KB200_IO);
        const bool ok = ::fstat(fd, &initial) == 0
                        && (directory ? S_ISDIR(initial.st_mode)
                                      : S_ISREG(initial.st_mode) && initial.st_size >= 24);
        if (!ok) {
            ::close(fd);
            fd = -1;
            raise("gguf_not_regular_file");
        }
    }
    File(File&& o) noexcept : fd(o.fd), initial(o.initial) {
        o.fd = -1;
    }
    File& operator=(File&&) = delete;
    File(const File&) = delete;
    ~File() {
        if (fd >= 0)
            ::close(fd);
    }

    uint64_t size() const {
        return uint64_t(initial.st_size);
    }

    void unchanged() const {
        struct stat now {};
        require(::fstat(fd, &now) == 0 && now.st_size == initial.st_size
                    && now.st_mtim.tv_sec == initial.st_mtim.tv_sec && now.st_mtim.tv_nsec == initial.st_mtim.tv_nsec
                    && now.st_ctim.tv_sec == initial.st_ctim.tv_sec && now.st_ctim.tv_nsec == initial.st_ctim.tv_nsec,
                "gguf_checkpoint_changed");
    }

    void read(uint64_t at, uint8_t* out, uint64_t n, const volatile uint8_t* cancel) const {
        require(at <= size() && n <= size() - at, "gguf_read_bounds");
        while (n) {
            stop(cancel);
            const ssize_t got = ::pread(fd, out, size_t(n), off_t(at));
            if (got < 0 && errno == EINTR)
                continue;
            if (got <= 0)
                raise("gguf_read_failed", KB200_IO);
            at += uint64_t(got), out += got, n -= uint64_t(got);
        }
    }
};

// Sequential little-endian reads of a header, through a 64 KiB window, never
// past the metadata limit or the end of the file.
class HeaderReader {
public:
    HeaderReader(const File& f, const volatile uint8_t* cancel) : file_(f), cancel_(cancel) {
    }

    uint64_t at() const {
        return at_;
    }

    void bytes(uint8_t* out, uint64_t n) {
        stop(cancel_);
        require(at_ <= kMetadataLimit && n <= kMetadataLimit - at_, "gguf_metadata_limit");
        require(n <= file_.size() - std::min(at_, file_.size()), "gguf_read_bounds");
        while (n) {
            if (at_ < begin_ || at_ >= begin_ + filled_) {
                begin_ = at_;
                filled_ = std::min<uint64_t>(sizeof(window_), file_.size() - at_);
                file_.read(at_, window_, filled_, cancel_);
            }
            const uint64_t take = std::min(n, begin_ + filled_ - at_);
            std::memcpy(out, window_ + (at_ - begin_), size_t(take));
            out += take, at_ += take, n -= take;
        }
    }

    void skip(uint64_t n) {
        stop(cancel_);
        require(at_ <= kMetadataLimit && n <= kMetadataLimit - at_ && n <= file_.size() - std::min(at_, file_.size()),
                "gguf_metadata_limit");
        at_ += n;
    }

    uint32_t u32() {
        uint8_t b[4];
        bytes(b, 4);
        return uint32_t(b[0]) | uint32_t(b[1]) << 8 | uint32_t(b[2]) << 16 | uint32_t(b[3]) << 24;
    }

    uint64_t u64() {
        uint8_t b[8];
        bytes(b, 8);
        uint64_t v = 0;
        for (int i = 7; i >= 0; --i)
            v = v << 8 | b[i];
        return v;
    }

    std::string text(uint64_t limit) {
        const uint64_t n = u64();
        require(n <= limit, "gguf_string_limit");
        std::string s(size_t(n), '\0');
        bytes(reinterpret_cast<uint8_t*>(&s[0]), n);
        require(s.find('\0') == std::string::npos, "gguf_string_nul");
        return s;
    }

private:
    const File& file_;
    const volatile uint8_t* cancel_;
    uint64_t at_ = 0, begin_ = 0, filled_ = 0;
    uint8_t window_[64 * 1024];
};

uint64_t type_width(uint32_t type) {
    switch (type) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: raise("gguf_metadata_type");
    }
}

// One metadata value as read: scalars widened, strings kept, numeric arrays
// kept as raw little-endian elements.
struct Value {
    uint32_t type = 0, element = 0;
    uint64_t count = 0;
    std::vector<uint8_t> raw;
    std::string text;
};

uint64_t raw_unsigned(const uint8_t* p, uint64_t width) {
    uint64_t v = 0;
    for (uint64_t i = width; i-- > 0;)
        v = v << 8 | p[i];
    return v;
}

int64_t raw_signed(const uint8_t* p, uint64_t width) {
    const uint64_t v = raw_unsigned(p, width), sign = uint64_t(1) << (8 * width - 1);
    return width == 8 ? int64_t(v) : int64_t(v ^ sign) - int64_t(sign);
}

double raw_float(const uint8_t* p, uint64_t width) {
    if (width == 4) {
        const uint32_t bits = uint32_t(raw_unsigned(p, 4));
        float f;
        std::memcpy(&f, &bits, 4);
        return f;
    }
    const uint64_t bits = raw_unsigned(p, 8);
    double d;
    std::memcpy(&d, &bits, 8);
    return d;
}

}  // namespace
}  // namespace kb200

namespace kb200 {
namespace {

struct TensorEntry {
    std::string name;
    uint64_t shape[3] = {1, 1, 1};
    uint32_t rank = 0, type = 0;
    int encoding = 0;
    uint32_t file = 0;
    uint64_t bytes = 0, row_bytes = 0, offset = 0, begin = 0;
};

struct Parsed {
    std::vector<TensorEntry> tensors;  // declaration order
    std::map<std::string, Value> kv;
    uint64_t header_end = 0, alignment = 32;
};

// One file's header: the reference's preflight (gguf_checkpoint.cpp:181-262)
// and then ggml's own layout rules (gguf.cpp), in that order of precedence.
Parsed parse_header(const File& f, const volatile uint8_t* cancel, uint32_t flags) {
    HeaderReader r(f, cancel);
    Parsed p;
    require(r.u32() == 0x46554747u && r.u32() == 3, "gguf_version");
    const uint64_t tensor_count = r.u64(), kv_count = r.u64();
    require(tensor_count <= kMaxTensors && kv_count <= kMaxKeys, "gguf_header_count");
    bool ggml_rejects = false;
    for (uint64_t i = 0; i < kv_count; ++i) {
        std::string key = r.text(256);
        require(p.kv.find(key) == p.kv.end(), "gguf_duplicate_key");
        ggml_rejects |= key.empty();
        Value v;
        v.type = r.u32();
        if (key == "general.alignment") {
            require(v.type == kU32, "gguf_alignment");
            const uint32_t a = r.u32();
            require(a && a <= 4096 && !(a & (a - 1)), "gguf_alignment");
            p.alignment = a;
            v.count = 1;
            v.raw = {uint8_t(a), uint8_t(a >> 8), uint8_t(a >> 16), uint8_t(a >> 24)};
        } else if (v.type == kString) {
            v.text = r.text(1 << 20);
            v.count = 1;
        } else if (v.type == kArray) {
            v.element = r.u32();
            v.count = r.u64();
            require(v.count <= kMaxArray && v.element != kArray, "gguf_array_limit");
            if (v.element == kString) {
                for (uint64_t k = 0; k < v.count; ++k)
                    (void)r.text(1 << 20);
            } else {
                const uint64_t n = mul(v.count, type_width(v.element));
                const uint64_t at = r.at();
                r.skip(n);
                v.raw.resize(size_t(n));
                if (n)
                    f.read(at, v.raw.data(), n, cancel);
            }
        } else {
            const uint64_t n = type_width(v.type);
            const uint64_t at = r.at();
            r.skip(n);
            v.raw.resize(size_t(n));
            f.read(at, v.raw.data(), n, cancel);
            v.count = 1;
        }
        p.kv.emplace(std::move(key), std::move(v));
    }
    std::map<std::string, int> names;
    for (uint64_t t = 0; t < tensor_count; ++t) {
        TensorEntry e;
        e.name = r.text(255);
        require(!e.name.empty() && names.emplace(e.name, 0).second, "gguf_duplicate_tensor");
        ggml_rejects |= e.name.size() >= kMaxName;
        e.rank = r.u32();
        require(e.rank >= 1 && e.rank <= 3, "gguf_tensor_rank");
        uint64_t rows = 1;
        for (uint32_t d = 0; d < e.rank; ++d) {
            e.shape[d] = r.u64();
            require(e.shape[d] && e.shape[d] <= uint64_t(INT64_MAX), "gguf_tensor_shape");
            if (d)
                rows = mul(rows, e.shape[d]);
        }
        e.type = r.u32();
        e.encoding = encoding_of(e.type, flags);
        require(e.encoding != -2, "gguf_tensor_type");
        const bool mx = e.encoding == KB200_GGUF_MXFP4;
        const uint64_t values = mx ? 32 : uint64_t(block_values(e.encoding));
        const uint64_t width = mx ? 17 : uint64_t(block_bytes(e.encoding));
        require(e.shape[0] % values == 0, "gguf_tensor_block_alignment");
        require(mul(e.shape[0], rows) <= uint64_t(INT64_MAX) && e.shape[0] <= SIZE_MAX / width, "gguf_tensor_shape");
        e.row_bytes = e.shape[0] / values * width;
        e.bytes = mul(e.row_bytes, rows);
        require(e.bytes <= uint64_t(INT64_MAX), "gguf_tensor_shape");
        e.offset = r.u64();
        p.tensors.push_back(std::move(e));
    }
    p.header_end = r.at();
    // ggml: tensors follow one another at the alignment from the aligned start
    // of the data section, which must lie inside the file.
    uint64_t data = p.header_end, running = 0;
    if (tensor_count) {
        data = (p.header_end + p.alignment - 1) / p.alignment * p.alignment;
        ggml_rejects |= data > f.size();
    }
    for (const auto& e : p.tensors) {
        ggml_rejects |= e.offset != running;
        if (e.bytes > UINT64_MAX - (p.alignment - 1))
            ggml_rejects = true;
        else
            running = add(running, (e.bytes + p.alignment - 1) / p.alignment * p.alignment);
    }
    if (ggml_rejects)
        raise("gguf_invalid_metadata");
    for (auto& e : p.tensors)
        e.begin = add(data, e.offset);
    return p;
}

const Value& metadata(const std::map<std::string, Value>& kv, const char* key) {
    require(key && std::strlen(key) <= 256, "gguf_metadata_key");
    const auto it = kv.find(key);
    require(it != kv.end(), "gguf_missing_metadata");
    return it->second;
}

// GgufCheckpoint::integer (gguf_checkpoint.cpp:384-408): unsigned 8-64 bit,
// or non-negative signed 32/64 bit.
uint64_t metadata_integer(const Value& v) {
    switch (v.type) {
    case kU8: case kU16: case kU32: case kU64:
        return raw_unsigned(v.raw.data(), type_width(v.type));
    case kI32: case kI64: {
        const int64_t s = raw_signed(v.raw.data(), type_width(v.type));
        require(s >= 0, "gguf_metadata_integer");
        return uint64_t(s);
    }
    default:
        raise("gguf_metadata_integer");
    }
}

// A numbered split name: <prefix>-NNNNN-of-NNNNN.gguf with a non-empty prefix.
bool split_name(const std::string& name, std::string& prefix, unsigned& number, unsigned& count) {
    static const char tail[] = "-00000-of-00000.gguf";
    const size_t n = sizeof(tail) - 1;
    if (name.size() <= n)
        return false;
    const std::string t = name.substr(name.size() - n);
    for (size_t i = 0; i < n; ++i) {
        const bool digit = tail[i] == '0';
        if (digit ? !(t[i] >= '0' && t[i] <= '9') : t[i] != tail[i])
            return false;
    }
    prefix = name.substr(0, name.size() - n);
    number = unsigned(std::stoul(t.substr(1, 5)));
    count = unsigned(std::stoul(t.substr(10, 5)));
    return true;
}

}  // namespace
}  // namespace kb200

struct kb200_gguf {
    std::vector<kb200::File> files;
    std::vector<kb200::TensorEntry> tensors;  // sorted by name
    std::map<std::string, kb200::Value> kv;   // the first file's metadata
};

namespace kb200 {
namespace {

const TensorEntry& find_tensor(const kb200_gguf* g, const char* name) {
    require(name != nullptr, "gguf_missing_tensor");
    const auto it = std::lower_bound(g->tensors.begin(), g->tensors.end(), name,
                                     [](const TensorEntry& e, const char* n) { return e.name < n; });
    require(it != g->tensors.end() && it->name == name, "gguf_missing_tensor");
    return *it;
}

void check_unchanged(const kb200_gguf* g) {
    for (const auto& f : g->files)
        f.unchanged();
}

// GgufCheckpoint::GgufCheckpoint (gguf_checkpoint.cpp:441-540).
kb200_gguf* open_root(const char* root, const volatile uint8_t* cancel, uint32_t flags) {
    require(root != nullptr, "gguf_missing_files");
    std::vector<std::string> names;
    {
        DIR* dir = ::opendir(root);
        if (!dir)
            raise("gguf_open_failed", KB200_IO);
        try {
            while (const dirent* d = ::readdir(dir)) {
                stop(cancel);
                const std::string n = d->d_name;
                if (n.size() > 5 && n.compare(n.size() - 5, 5, ".gguf") == 0)
                    names.push_back(n);
                require(names.size() <= 512, "gguf_split_count");
            }
        } catch (...) {
            ::closedir(dir);
            throw;
        }
        ::closedir(dir);
    }
    require(!names.empty(), "gguf_missing_files");
    std::sort(names.begin(), names.end());
    File directory(::open(root, O_RDONLY | O_DIRECTORY | O_NOFOLLOW | O_CLOEXEC), true);
    std::string prefix0, prefix;
    unsigned number = 0, count = 0;
    const bool single = names.size() == 1 && !split_name(names[0], prefix, number, count);
    auto* g = new kb200_gguf;
    try {
        uint64_t total = 0, metadata_bytes = 0;
        for (size_t i = 0; i < names.size(); ++i) {
            const bool matched = split_name(names[i], prefix, number, count);
            require(names[i].size() <= 255 && (single || matched), "gguf_split_name");
            if (!single && i == 0)
                prefix0 = prefix;
            require(single || (prefix == prefix0 && number == i + 1 && count == names.size()), "gguf_split_name");
            g->files.emplace_back(::openat(directory.fd, names[i].c_str(), O_RDONLY | O_NOFOLLOW | O_CLOEXEC), false);
            const File& file = g->files.back();
            Parsed p = parse_header(file, cancel, flags);
            metadata_bytes = add(metadata_bytes, p.header_end);
            require(metadata_bytes <= kSplitMetadataLimit, "gguf_metadata_limit");
            file.unchanged();
            if (!single) {
                require(metadata_integer(metadata(p.kv, "split.no")) == i
                            && metadata_integer(metadata(p.kv, "split.count")) == names.size(),
                        "gguf_split_metadata");
            }
            const uint64_t expected =
                single ? p.tensors.size() : metadata_integer(metadata(p.kv, "split.tensors.count"));
            if (i == 0)
                total = expected;
            require(expected == total && total <= kMaxTensors, "gguf_split_metadata");
            for (auto& e : p.tensors) {
                require(e.offset % p.alignment == 0 && add(e.begin, e.bytes) <= file.size(), "gguf_tensor_bounds");
                e.file = uint32_t(i);
                g->tensors.push_back(std::move(e));
            }
            file.unchanged();
            if (i == 0)
                g->kv = std::move(p.kv);
        }
        require(g->tensors.size() == total, "gguf_tensor_count");
        std::sort(g->tensors.begin(), g->tensors.end(),
                  [](const TensorEntry& a, const TensorEntry& b) { return a.name < b.name; });
        for (size_t i = 1; i < g->tensors.size(); ++i)
            require(g->tensors[i - 1].name != g->tensors[i].name, "gguf_duplicate_tensor");
        check_unchanged(g);
    } catch (...) {
        delete g;
        throw;
    }
    return g;
}

// GgufCheckpoint::read_packed_rows (gguf_checkpoint.cpp:644-674).
void read_rows(const kb200_gguf* g, const TensorEntry& t, uint64_t expert, uint64_t first_row, void* output,
               uint64_t bytes, const volatile uint8_t* cancel) {
    stop(cancel);
    require(t.rank >= 2 && expert < t.shape[2] && bytes % t.row_bytes == 0 && first_row <= t.shape[1]
                && bytes / t.row_bytes <= t.shape[1] - first_row,
            "gguf_row_range");
    require(output != nullptr || bytes == 0, "gguf_row_range");
    const File& file = g->files[t.file];
    file.unchanged();
    const uint64_t offset = add(t.begin, mul(add(mul(expert, t.shape[1]), first_row), t.row_bytes));
    auto* out = static_cast<uint8_t*>(output);
    for (uint64_t at = 0; at < bytes; at += kReadPiece) {
        stop(cancel);
        file.read(add(offset, at), out + at, std::min(kReadPiece, bytes - at), cancel);
    }
    file.unchanged();
    stop(cancel);
}

void describe(const TensorEntry& t, kb200_gguf_tensor* info) {
    for (int d = 0; d < 3; ++d)
        info->shape[d] = t.shape[d];
    info->rank = t.rank;
    info->ggml_type = t.type;
    info->encoding = t.encoding;
    info->file = t.file;
    info->bytes = t.bytes;
    info->row_bytes = t.row_bytes;
    info->offset = t.begin;
}

// Runs `body`, turning a reader failure into its status and message.
template <class F>
int guarded(F&& body) {
    try {
        body();
        return KB200_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.what);
    } catch (const std::bad_alloc&) {
        return fail(KB200_NO_MEMORY, "gguf_metadata_memory");
    } catch (const std::exception& e) {
        return fail(KB200_INVALID, e.what());
    }
}

}  // namespace
}  // namespace kb200

using namespace kb200;

extern "C" {

int kb200_gguf_open(const char* root, const volatile uint8_t* cancel, kb200_gguf** out) {
    return kb200_gguf_open_flags(root, cancel, 0, out);
}

int kb200_gguf_open_flags(const char* root, const volatile uint8_t* cancel, uint32_t flags, kb200_gguf** out) {
    if (!out)
        return fail(KB200_INVALID, "null output");
    *out = nullptr;
    if (flags & ~uint32_t(KB200_GGUF_ACCEPT_MXFP4))
        return fail(KB200_INVALID, "unknown GGUF open flags");
    return guarded([&] { *out = open_root(root, cancel, flags); });
}

void kb200_gguf_close(kb200_gguf* g) {
    delete g;
}

size_t kb200_gguf_tensor_count(const kb200_gguf* g) {
    return g ? g->tensors.size() : 0;
}

int kb200_gguf_tensor_at(const kb200_gguf* g, size_t index, kb200_gguf_tensor* info, const char** name) {
    if (!g || !info)
        return fail(KB200_INVALID, "null checkpoint or info");
    if (index >= g->tensors.size())
        return fail(KB200_INVALID, "gguf_tensor_index");
    describe(g->tensors[index], info);
    if (name)
        *name = g->tensors[index].name.c_str();
    return KB200_OK;
}

int kb200_gguf_find_tensor(const kb200_gguf* g, const char* name, kb200_gguf_tensor* info) {
    if (!g || !info)
        return fail(KB200_INVALID, "null checkpoint or info");
    return guarded([&] { describe(find_tensor(g, name), info); });
}

// GgufCheckpoint::identity (gguf_checkpoint.cpp:566-588).
int kb200_gguf_identity(const kb200_gguf* g, const char* name, uint64_t expert, kb200_weight_identity* id) {
    if (!g || !id)
        return fail(KB200_INVALID, "null checkpoint or identity");
    return guarded([&] {
        const TensorEntry& t = find_tensor(g, name);
        require(expert < t.shape[2], "gguf_expert_range");
        const File& file = g->files[t.file];
        file.unchanged();
        const struct stat& s = file.initial;
        const uint64_t per_expert = t.bytes / t.shape[2], begin = add(t.begin, mul(expert, per_expert));
        *id = kb200_weight_identity{uint64_t(s.st_dev), uint64_t(s.st_ino), uint64_t(s.st_size),
                                    uint64_t(s.st_mtim.tv_sec), uint64_t(s.st_mtim.tv_nsec),
                                    uint64_t(s.st_ctim.tv_sec), uint64_t(s.st_ctim.tv_nsec),
                                    begin, add(begin, per_expert)};
    });
}

int kb200_gguf_check_unchanged(const kb200_gguf* g) {
    if (!g)
        return fail(KB200_INVALID, "null checkpoint");
    return guarded([&] { check_unchanged(g); });
}

int kb200_gguf_read_packed_rows(const kb200_gguf* g, const char* name, uint64_t expert, uint64_t first_row,
                                void* output, uint64_t bytes, const volatile uint8_t* cancel) {
    if (!g)
        return fail(KB200_INVALID, "null checkpoint");
    return guarded([&] { read_rows(g, find_tensor(g, name), expert, first_row, output, bytes, cancel); });
}

// GgufCheckpoint::read_vector (gguf_checkpoint.cpp:676-701).
int kb200_gguf_read_vector(const kb200_gguf* g, const char* name, float* output, uint64_t count,
                           const volatile uint8_t* cancel) {
    if (!g)
        return fail(KB200_INVALID, "null checkpoint");
    return guarded([&] {
        stop(cancel);
        const TensorEntry& t = find_tensor(g, name);
        require(t.type == 0 && count == t.shape[0] * t.shape[1] * t.shape[2] && count * sizeof(float) == t.bytes,
                "gguf_vector_shape");
        require(output != nullptr || count == 0, "gguf_vector_shape");
        const File& file = g->files[t.file];
        file.unchanged();
        auto* raw = reinterpret_cast<uint8_t*>(output);
        for (uint64_t at = 0; at < t.bytes; at += 65536) {
            stop(cancel);
            file.read(add(t.begin, at), raw + at, std::min<uint64_t>(65536, t.bytes - at), nullptr);
        }
        for (uint64_t i = 0; i < count; ++i)
            require(std::isfinite(output[i]), "gguf_nonfinite_weight");
        file.unchanged();
        stop(cancel);
    });
}

int kb200_gguf_has(const kb200_gguf* g, const char* key) {
    return g && key && std::strlen(key) <= 256 && g->kv.count(key) ? 1 : 0;
}

int kb200_gguf_integer(const kb200_gguf* g, const char* key, uint64_t* value) {
    if (!g || !value)
        return fail(KB200_INVALID, "null checkpoint or value");
    return guarded([&] { *value = metadata_integer(metadata(g->kv, key)); });
}

// GgufCheckpoint::number (gguf_checkpoint.cpp:711-720): floats, or an integer as above; finite.
int kb200_gguf_number(const kb200_gguf* g, const char* key, double* value) {
    if (!g || !value)
        return fail(KB200_INVALID, "null checkpoint or value");
    return guarded([&] {
        const Value& v = metadata(g->kv, key);
        const double d = v.type == kF32 || v.type == kF64 ? raw_float(v.raw.data(), type_width(v.type))
                                                          : double(metadata_integer(v));
        require(std::isfinite(d), "gguf_metadata_number");
        *value = d;
    });
}

int kb200_gguf_boolean(const kb200_gguf* g, const char* key, int* value) {
    if (!g || !value)
        return fail(KB200_INVALID, "null checkpoint or value");
    return guarded([&] {
        const Value& v = metadata(g->kv, key);
        require(v.type == kBool, "gguf_metadata_boolean");
        *value = v.raw[0] != 0;
    });
}

int kb200_gguf_string(const kb200_gguf* g, const char* key, const char** value, size_t* length) {
    if (!g || !value)
        return fail(KB200_INVALID, "null checkpoint or value");
    return guarded([&] {
        const Value& v = metadata(g->kv, key);
        require(v.type == kString, "gguf_metadata_string");
        *value = v.text.c_str();
        if (length)
            *length = v.text.size();
    });
}

// GgufCheckpoint::integers (gguf_checkpoint.cpp:726-752).
int kb200_gguf_integers(const kb200_gguf* g, const char* key, int64_t* values, size_t capacity, size_t* count) {
    if (!g || !count || (capacity && !values))
        return fail(KB200_INVALID, "null checkpoint or values");
    return guarded([&] {
        const Value& v = metadata(g->kv, key);
        require(v.type == kArray, "gguf_metadata_integers");
        require(v.count <= kMaxArray, "gguf_array_limit");
        require(v.element == kI32 || v.element == kU32 || v.element == kI64 || v.element == kU64,
                "gguf_metadata_integers");
        const uint64_t w = type_width(v.element);
        std::vector<int64_t> out(size_t(v.count));
        for (uint64_t i = 0; i < v.count; ++i) {
            const uint8_t* p = v.raw.data() + i * w;
            if (v.element == kU64) {
                const uint64_t u = raw_unsigned(p, 8);
                require(u <= uint64_t(INT64_MAX), "gguf_metadata_integers");
                out[i] = int64_t(u);
            } else if (v.element == kU32) {
                out[i] = int64_t(raw_unsigned(p, 4));
            } else {
                out[i] = raw_signed(p, w);
            }
        }
        *count = out.size();
        std::copy_n(out.begin(), std::min(out.size(), capacity), values);
    });
}

// GgufCheckpoint::numbers (gguf_checkpoint.cpp:754-767): float32 arrays, finite.
int kb200_gguf_numbers(const kb200_gguf* g, const char* key, double* values, size_t capacity, size_t* count) {
    if (!g || !count || (capacity && !values))
        return fail(KB200_INVALID, "null checkpoint or values");
    return guarded([&] {
        const Value& v = metadata(g->kv, key);
        require(v.type == kArray && v.element == kF32, "gguf_metadata_numbers");
        require(v.count <= kMaxArray, "gguf_array_limit");
        std::vector<double> out(size_t(v.count));
        for (uint64_t i = 0; i < v.count; ++i) {
            out[i] = raw_float(v.raw.data() + i * 4, 4);
            require(std::isfinite(out[i]), "gguf_metadata_numbers");
        }
        *count = out.size();
        std::copy_n(out.begin(), std::min(out.size(), capacity), values);
    });
}

int kb200_gguf_rows_bind(const kb200_gguf* g, const char* name, uint64_t expert, kb200_gguf_rows* rows) {
    if (!g || !rows)
        return fail(KB200_INVALID, "null checkpoint or rows");
    return guarded([&] {
        const TensorEntry& t = find_tensor(g, name);
        require(t.rank >= 2, "gguf_row_range");
        require(expert < t.shape[2], "gguf_expert_range");
        *rows = kb200_gguf_rows{g, uint64_t(&t - g->tensors.data()), expert};
    });
}

int kb200_gguf_rows_source(void* user, uint64_t first_row, void* dst, uint64_t bytes) {
    const auto* rows = static_cast<const kb200_gguf_rows*>(user);
    if (!rows || !rows->file || rows->tensor >= rows->file->tensors.size())
        return fail(KB200_INVALID, "unbound packed-row source");
    return guarded([&] {
        read_rows(rows->file, rows->file->tensors[size_t(rows->tensor)], rows->expert, first_row, dst, bytes,
                  nullptr);
    });
}

}  // extern "C"

// Safetensors shard reader: the reference worker's kadan::checkpoint::Shard
// (services/hikari/inference_worker/src/weights/checkpoint.cpp:449-730) for the
// gpt-oss MXFP4 expert tensors the MoE layer consumes.
//
// A safetensors file is an 8-byte little-endian header length, a JSON object
// mapping tensor names to {dtype, shape, data_offsets} (plus an optional
// "__metadata__" object of strings), then the payload. The header is read by
// a token cursor (lexical checks as each token is taken) driving one generic
// sequence reader and small rule tables (descriptor fields, dtype names), so
// the schema is data rather than code. Accepted exactly when the reference
// accepts: ASCII strings and escapes, unsigned decimal integers, exactly the
// three descriptor fields, and tensors that tile the payload with no gap or
// overlap; failures carry the reference's messages, checked against its own
// reader on malformed and randomly mutated files.
#include <algorithm>
#include <cerrno>
#include <cstdint>
#include <cstring>
#include <fcntl.h>
#include <limits>
#include <new>
#include <string>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>

#include "kb200_host.hpp"

namespace kb200 {
namespace st {
namespace {

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
    require(b <= UINT64_MAX - a, "size_overflow");
    return a + b;
}

uint64_t mul(uint64_t a, uint64_t b) {
    require(b == 0 || a <= UINT64_MAX / b, "size_overflow");
    return a * b;
}

struct stat regular_file(int fd) {
    struct stat s {};
    if (::fstat(fd, &s) != 0)
        raise("stat_failed", KB200_IO);
    require(S_ISREG(s.st_mode) && s.st_size >= 8, "not_safetensors_file");
    return s;
}

void read_at(int fd, uint64_t offset, uint8_t* out, uint64_t n) {
    require(add(offset, n) <= uint64_t(std::numeric_limits<off_t>::max()), "file_offset_overflow");
    while (n) {
        const uint64_t piece = std::min<uint64_t>(n, 1u << 20);
        const ssize_t got = ::pread(fd, out, size_t(piece), off_t(offset));
        if (got < 0 && errno == EINTR)
            continue;
        if (got <= 0)
            raise("short_or_failed_read", KB200_IO);
        offset += uint64_t(got), out += got, n -= uint64_t(got);
    }
}

// A shard basename: 1-255 characters of [A-Za-z0-9._-], not "." or "..".
void basename(const std::string& name) {
    require(!name.empty() && name.size() <= 255 && name != "." && name != "..", "invalid_shard_name");
    for (const unsigned char c : name)
        require((c >= 'a' && c <= 'z') || (c >= 'A' && c <= 'Z') || (c >= '0' && c <= '9') || c == '.' || c == '_'
                    || c == '-',
                "invalid_shard_name");
}

struct Tensor {
    std::string name;
    int dtype = 0;
    uint64_t shape[8] = {};
    uint32_t rank = 0;
    uint64_t begin = 0, end = 0;

    uint64_t elements() const {
        uint64_t n = 1;
        for (uint32_t i = 0; i < rank; ++i)
            n = mul(n, shape[i]);
        return n;
    }
};

uint64_t dtype_width(int dtype) {
    return dtype == KB200_DTYPE_F32 || dtype == KB200_DTYPE_U32   ? 4
           : dtype == KB200_DTYPE_BF16 || dtype == KB200_DTYPE_F16 ? 2
                                                                   : 1;
}

// ---------------------------------------------------------------- lexical
// A cursor over the header text that hands out JSON tokens on demand: blanks
// are skipped before every punctuation mark, string or number, and each token
// is checked as it is taken, so a malformed header fails at the first token
// that breaks the schema, in text order.
class Cursor {
public:
    Cursor(const char* text, size_t size) : at_(text), end_(text + size) {}

    // The next significant character is `c`: consume it.
    bool eat(char c) {
        blanks();
        if (at_ == end_ || *at_ != c)
            return false;
        ++at_;
        return true;
    }

    void need(char c) { require(eat(c), "json_syntax"); }

    // Nothing but blanks is left.
    bool finished() {
        blanks();
        return at_ == end_;
    }

    // A quoted ASCII string of at most `limit` characters after unescaping.
    std::string quoted(uint64_t limit) {
        need('"');
        std::string out;
        for (;;) {
            require(at_ != end_, "unterminated_string");
            const unsigned char raw = static_cast<unsigned char>(*at_++);
            if (raw == '"')
                return out;
            require(raw >= 0x20 && raw < 0x80, "non_ascii_json_string");
            const char c = raw == '\\' ? escaped() : char(raw);
            require(out.size() < limit, "json_string_limit");
            out.push_back(c);
        }
    }

    // An unsigned decimal integer: digits only, no leading zero, fits 64 bits.
    uint64_t natural() {
        blanks();
        const char* first = at_;
        uint64_t value = 0;
        bool overflow = false;
        for (; at_ != end_ && *at_ >= '0' && *at_ <= '9'; ++at_) {
            const uint64_t digit = uint64_t(*at_ - '0');
            overflow |= value > (UINT64_MAX - digit) / 10;
            value = value * 10 + digit;
        }
        const size_t digits = size_t(at_ - first);
        require(digits != 0 && !(digits > 1 && *first == '0') && !overflow, "json_integer");
        return value;
    }

private:
    void blanks() {
        while (at_ != end_ && (*at_ == ' ' || *at_ == '\t' || *at_ == '\n' || *at_ == '\r'))
            ++at_;
    }

    // The character a backslash sequence stands for (the backslash is taken).
    char escaped() {
        // Single-letter escapes: the letter and what it stands for.
        static constexpr char kSimple[][2] = {{'"', '"'}, {'\\', '\\'}, {'/', '/'}, {'b', '\b'},
                                              {'f', '\f'}, {'n', '\n'}, {'r', '\r'}, {'t', '\t'}};
        require(at_ != end_, "json_escape");
        const char letter = *at_++;
        for (const auto& e : kSimple)
            if (e[0] == letter)
                return e[1];
        require(letter == 'u', "json_escape");
        unsigned code = 0;
        for (int i = 0; i < 4; ++i) {
            require(at_ != end_, "json_escape");
            const int nibble = hex_value(*at_++);
            require(nibble >= 0, "json_escape");
            code = code << 4 | unsigned(nibble);
        }
        // Only \u0001..\u007f: names and values are ASCII.
        require(code - 1u < 0x7fu, "non_ascii_json_string");
        return char(code);
    }

    static int hex_value(char c) {
        if (c >= '0' && c <= '9')
            return c - '0';
        const char lower = char(c | 0x20);
        return lower >= 'a' && lower <= 'f' ? lower - 'a' + 10 : -1;
    }

    const char* at_;
    const char* end_;
};

// ----------------------------------------------------------------- schema
// `open` member (`,` member)* `close`, or `open close` when empty is allowed;
// `each` reads one member.
template <class Each>
void sequence(Cursor& c, char open, char close, bool may_be_empty, Each&& each) {
    c.need(open);
    if (may_be_empty && c.eat(close))
        return;
    do
        each();
    while (c.eat(','));
    c.need(close);
}

constexpr uint64_t kNameLimit = 512;     // tensor names, metadata keys, field names
constexpr size_t kMetadataKeys = 1024;

struct DtypeName {
    const char* text;
    int dtype;
};
constexpr DtypeName kDtypes[] = {{"U8", KB200_DTYPE_U8},           {"U32", KB200_DTYPE_U32},
                                 {"I8", KB200_DTYPE_I8},           {"F8_E4M3", KB200_DTYPE_F8_E4M3},
                                 {"F32", KB200_DTYPE_F32},         {"F16", KB200_DTYPE_F16},
                                 {"BF16", KB200_DTYPE_BF16}};

void read_dtype(Cursor& c, Tensor& t) {
    const std::string name = c.quoted(kNameLimit);
    for (const auto& d : kDtypes)
        if (name == d.text) {
            t.dtype = d.dtype;
            return;
        }
    raise("unsupported_dtype");
}

void read_shape(Cursor& c, Tensor& t) {
    sequence(c, '[', ']', true, [&] {
        require(t.rank < 8, "rank_limit");
        t.shape[t.rank++] = c.natural();
    });
}

void read_offsets(Cursor& c, Tensor& t) {
    c.need('[');
    t.begin = c.natural();
    c.need(',');
    t.end = c.natural();
    c.need(']');
}

// The three descriptor fields, each exactly once, in any order.
struct FieldRule {
    const char* key;
    unsigned bit;
    void (*read)(Cursor&, Tensor&);
};
constexpr FieldRule kFields[] = {{"dtype", 1u, read_dtype}, {"shape", 2u, read_shape},
                                 {"data_offsets", 4u, read_offsets}};
constexpr unsigned kAllFields = 7u;

void read_descriptor(Cursor& c, Tensor& t) {
    unsigned seen = 0;
    sequence(c, '{', '}', false, [&] {
        const std::string key = c.quoted(kNameLimit);
        c.need(':');
        const FieldRule* rule = nullptr;
        for (const auto& f : kFields)
            if (key == f.key)
                rule = &f;
        if (!rule)
            raise("unknown_tensor_field");
        rule->read(c, t);
        require(!(seen & rule->bit), "duplicate_tensor_field");
        seen |= rule->bit;
    });
    require(seen == kAllFields, "missing_tensor_field");
    require(t.end >= t.begin && t.end - t.begin == mul(t.elements(), dtype_width(t.dtype)), "tensor_byte_size");
}

void read_metadata(Cursor& c, uint64_t value_limit) {
    std::vector<std::string> keys;
    sequence(c, '{', '}', true, [&] {
        std::string key = c.quoted(kNameLimit);
        require(keys.size() < kMetadataKeys && std::find(keys.begin(), keys.end(), key) == keys.end(),
                "metadata_key_limit_or_duplicate");
        keys.push_back(std::move(key));
        c.need(':');
        (void)c.quoted(value_limit);
    });
}

// The whole header: one object of tensor descriptors and at most one
// "__metadata__" object, nothing after it but blanks.
void read_header(const char* text, size_t size, uint64_t metadata_limit, uint64_t tensor_limit,
                 std::vector<Tensor>& tensors) {
    require(size != 0 && text[0] == '{', "header_start");
    Cursor c(text, size);
    bool metadata = false;
    sequence(c, '{', '}', true, [&] {
        std::string name = c.quoted(kNameLimit);
        c.need(':');
        if (name == "__metadata__") {
            require(!metadata, "duplicate_metadata");
            metadata = true;
            read_metadata(c, metadata_limit);
            return;
        }
        require(!name.empty() && tensors.size() < tensor_limit, "tensor_limit_or_name");
        Tensor t;
        t.name = std::move(name);
        read_descriptor(c, t);
        tensors.push_back(std::move(t));
    });
    require(c.finished(), "trailing_json");
}

}  // namespace
}  // namespace st
}  // namespace kb200

struct kb200_shard {
    int fd = -1;
    struct stat identity {};
    uint64_t data_begin = 0;
    std::vector<kb200::st::Tensor> tensors;  // sorted by name
    ~kb200_shard() {
        if (fd >= 0)
            ::close(fd);
    }
};

namespace kb200 {
namespace st {
namespace {

void unchanged(const kb200_shard* s) {
    const struct stat now = regular_file(s->fd);
    const struct stat& was = s->identity;
    require(now.st_size == was.st_size && now.st_mtim.tv_sec == was.st_mtim.tv_sec
                && now.st_mtim.tv_nsec == was.st_mtim.tv_nsec && now.st_ctim.tv_sec == was.st_ctim.tv_sec
                && now.st_ctim.tv_nsec == was.st_ctim.tv_nsec,
            "checkpoint_changed");
}

const Tensor& find(const kb200_shard* s, const char* name) {
    require(name != nullptr, "missing_tensor");
    const auto it = std::lower_bound(s->tensors.begin(), s->tensors.end(), name,
                                     [](const Tensor& t, const char* n) { return t.name < n; });
    require(it != s->tensors.end() && it->name == name, "missing_tensor");
    return *it;
}

void read(const kb200_shard* s, const Tensor& t, uint64_t skip, uint8_t* out, uint64_t n) {
    require(skip <= t.end - t.begin && n <= t.end - t.begin - skip, "tensor_read_bounds");
    read_at(s->fd, add(s->data_begin, add(t.begin, skip)), out, n);
}

// Shard::Shard (checkpoint.cpp:449-511).
kb200_shard* open_shard(const char* root, const char* shard_name, const kb200_shard_limits* given) {
    kb200_shard_limits limits{16u << 20, 65536, 512};
    if (given)
        limits = *given;
    require(limits.header_bytes != 0 && limits.tensors != 0, "invalid_reader_limits");
    require(root != nullptr && shard_name != nullptr, "invalid_shard_name");
    const std::string name(shard_name);
    basename(name);
    const int dir = ::open(root, O_RDONLY | O_DIRECTORY | O_NOFOLLOW | O_CLOEXEC);
    if (dir < 0)
        raise("open_failed", KB200_IO);
    const int fd = ::openat(dir, name.c_str(), O_RDONLY | O_NOFOLLOW | O_NONBLOCK | O_CLOEXEC);
    ::close(dir);
    if (fd < 0)
        raise("open_failed", KB200_IO);
    auto* s = new kb200_shard;
    s->fd = fd;
    try {
        s->identity = regular_file(fd);
        uint8_t prefix[8];
        read_at(fd, 0, prefix, 8);
        uint64_t header_size = 0;
        for (int i = 7; i >= 0; --i)
            header_size = header_size << 8 | prefix[i];
        require(header_size > 0 && header_size <= limits.header_bytes
                    && header_size <= uint64_t(s->identity.st_size) - 8,
                "header_size");
        s->data_begin = add(8, header_size);
        std::vector<char> text(static_cast<size_t>(header_size));
        read_at(fd, 8, reinterpret_cast<uint8_t*>(text.data()), header_size);
        read_header(text.data(), text.size(), limits.metadata_value_bytes, limits.tensors, s->tensors);
        auto& t = s->tensors;
        std::sort(t.begin(), t.end(),
                  [](const Tensor& a, const Tensor& b) { return a.begin == b.begin ? a.end < b.end : a.begin < b.begin; });
        uint64_t previous = 0;
        for (const auto& x : t) {
            require(x.begin == previous, "tensor_gap_or_overlap");
            previous = x.end;
        }
        require(previous == uint64_t(s->identity.st_size) - s->data_begin, "payload_coverage");
        std::sort(t.begin(), t.end(), [](const Tensor& a, const Tensor& b) { return a.name < b.name; });
        for (size_t i = 1; i < t.size(); ++i)
            require(t[i - 1].name != t[i].name, "duplicate_tensor");
        unchanged(s);
    } catch (...) {
        delete s;
        throw;
    }
    return s;
}

void describe(const kb200_shard* s, const Tensor& t, kb200_shard_tensor* info) {
    for (int d = 0; d < 8; ++d)
        info->shape[d] = t.shape[d];
    info->rank = t.rank;
    info->dtype = t.dtype;
    info->bytes = t.end - t.begin;
    info->offset = s->data_begin + t.begin;
}

template <class F>
int guarded(F&& body) {
    try {
        body();
        return KB200_OK;
    } catch (const Failure& f) {
        return fail(f.status, f.what);
    } catch (const std::bad_alloc&) {
        return fail(KB200_NO_MEMORY, "checkpoint_metadata_memory");
    } catch (const std::exception& e) {
        return fail(KB200_INVALID, e.what());
    }
}

}  // namespace
}  // namespace st
}  // namespace kb200

using namespace kb200;
using namespace kb200::st;

extern "C" {

int kb200_shard_open(const char* root, const char* name, const kb200_shard_limits* limits, kb200_shard** out) {
    if (!out)
        return fail(KB200_INVALID, "null output");
    *out = nullptr;
    return guarded([&] { *out = open_shard(root, name, limits); });
}

void kb200_shard_close(kb200_shard* s) {
    delete s;
}

size_t kb200_shard_tensor_count(const kb200_shard* s) {
    return s ? s->tensors.size() : 0;
}

int kb200_shard_tensor_at(const kb200_shard* s, size_t index, kb200_shard_tensor* info, const char** name) {
    if (!s || !info)
        return fail(KB200_INVALID, "null shard or info");
    if (index >= s->tensors.size())
        return fail(KB200_INVALID, "tensor_index");
    describe(s, s->tensors[index], info);
    if (name)
        *name = s->tensors[index].name.c_str();
    return KB200_OK;
}

int kb200_shard_find_tensor(const kb200_shard* s, const char* name, kb200_shard_tensor* info) {
    if (!s || !info)
        return fail(KB200_INVALID, "null shard or info");
    return guarded([&] { describe(s, find(s, name), info); });
}

// Shard::tensor_identity (checkpoint.cpp:539-553).
int kb200_shard_identity(const kb200_shard* s, const char* name, kb200_weight_identity* id) {
    if (!s || !id)
        return fail(KB200_INVALID, "null shard or identity");
    return guarded([&] {
        const Tensor& t = find(s, name);
        const struct stat& st = s->identity;
        *id = kb200_weight_identity{uint64_t(st.st_dev), uint64_t(st.st_ino), uint64_t(st.st_size),
                                    uint64_t(st.st_mtim.tv_sec), uint64_t(st.st_mtim.tv_nsec),
                                    uint64_t(st.st_ctim.tv_sec), uint64_t(st.st_ctim.tv_nsec),
                                    s->data_begin + t.begin, s->data_begin + t.end};
    });
}

int kb200_shard_check_unchanged(const kb200_shard* s) {
    if (!s)
        return fail(KB200_INVALID, "null shard");
    return guarded([&] { unchanged(s); });
}

// Shard::read_tensor (checkpoint.cpp:560-580), without the shared read cache.
int kb200_shard_read_tensor(const kb200_shard* s, const char* name, uint64_t offset, void* output, uint64_t bytes) {
    if (!s || (bytes && !output))
        return fail(KB200_INVALID, "null shard or output");
    return guarded([&] {
        const Tensor& t = find(s, name);
        unchanged(s);
        read(s, t, offset, static_cast<uint8_t*>(output), bytes);
        unchanged(s);
    });
}

// Shard::load_mxfp4_expert_rows (checkpoint.cpp:669-730) and the MXFP4 check
// of quantization::validate (quantization.cpp:45-54): no scale byte is 255.
int kb200_shard_load_mxfp4_expert_rows(const kb200_shard* s, const char* prefix, uint64_t expert, uint64_t first,
                                       uint64_t count, uint64_t payload_budget, void* weights,
                                       uint64_t weights_capacity, void* scales, uint64_t scales_capacity,
                                       uint64_t* columns) {
    if (!s)
        return fail(KB200_INVALID, "null shard");
    return guarded([&] {
        const size_t plen = prefix ? std::strlen(prefix) : 0;
        require(plen != 0 && plen <= 480 && count != 0, "projection_range_or_name");
        const Tensor& blocks = find(s, (std::string(prefix) + "_blocks").c_str());
        const Tensor& sc = find(s, (std::string(prefix) + "_scales").c_str());
        require(blocks.dtype == KB200_DTYPE_U8 && sc.dtype == KB200_DTYPE_U8, "mxfp4_dtype");
        require(blocks.rank == 4 && sc.rank == 3 && blocks.shape[3] == 16 && blocks.shape[2] > 0
                    && expert < blocks.shape[0] && first <= blocks.shape[1] && count <= blocks.shape[1] - first
                    && std::equal(sc.shape, sc.shape + 3, blocks.shape),
                "mxfp4_expert_shape");
        const uint64_t groups = blocks.shape[2];
        const uint64_t scale_bytes = mul(count, groups), weight_bytes = mul(scale_bytes, 16);
        const uint64_t cols = mul(groups, 32), total = add(weight_bytes, scale_bytes);
        const uint64_t scale_offset = mul(add(mul(expert, blocks.shape[1]), first), groups);
        const uint64_t weight_offset = mul(scale_offset, 16);
        require(total <= payload_budget, "payload_budget");
        require(weights && scales && weights_capacity >= weight_bytes && scales_capacity >= scale_bytes,
                "output_capacity");
        unchanged(s);
        read(s, blocks, weight_offset, static_cast<uint8_t*>(weights), weight_bytes);
        read(s, sc, scale_offset, static_cast<uint8_t*>(scales), scale_bytes);
        unchanged(s);
        const auto* e8m0 = static_cast<const uint8_t*>(scales);
        require(std::find(e8m0, e8m0 + scale_bytes, uint8_t(255)) == e8m0 + scale_bytes, "invalid_block_scale");
        if (columns)
            *columns = cols;
    });
}

}  // extern "C"

// Read-fault injection for the checkpoint readers (kadan_b200/csrc/gguf_file.cpp
// and safetensors.cpp), the way the reference tests its GGUF reader: pread is
// wrapped at link time (-Wl,--wrap=pread). Short reads and an interrupted read
// must not change what is read; an I/O error at any read of opening or of a row
// read must fail that call with KB200_IO and the reference's message.
//
//   reader_faults_test <gguf dir> <tensor> <rows file> <shard dir> <shard> <prefix> <rows file>
//
// The rows files hold the bytes expected for all rows of expert 0. Prints "ok".
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <iterator>
#include <string>
#include <sys/types.h>
#include <vector>

#include "kadan_b200.h"
#include "kb200_host.hpp"

namespace kb200 {
namespace {
char last_error[512];
}
// The library records failures through these; the harness keeps the text.
int fail(int status, const char* what) {
    std::snprintf(last_error, sizeof(last_error), "%s", what);
    return status;
}
int cuda_fail(cudaError_t, const char* where) {
    std::snprintf(last_error, sizeof(last_error), "cuda: %s", where);
    return KB200_CUDA;
}
}  // namespace kb200

namespace {

enum class Mode { pass, short_reads, interrupt_once, fail_at };
Mode mode = Mode::pass;
long fail_at = -1, calls = 0;
bool interrupted = false;

void set(Mode m, long at = -1) {
    mode = m, fail_at = at, calls = 0, interrupted = false;
}

std::vector<char> slurp(const char* path) {
    std::ifstream f(path, std::ios::binary);
    return {std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>()};
}

#define CHECK(c)                                                                       \
    do {                                                                               \
        if (!(c)) {                                                                    \
            std::fprintf(stderr, "%s:%d: check failed: %s (last error: %s)\n", __FILE__, \
                         __LINE__, #c, kb200::last_error);                             \
            std::exit(1);                                                              \
        }                                                                              \
    } while (0)

}  // namespace

extern "C" ssize_t __real_pread(int fd, void* buf, size_t n, off_t offset);
extern "C" ssize_t __wrap_pread(int fd, void* buf, size_t n, off_t offset) {
    const long call = calls++;
    if (mode == Mode::fail_at && call == fail_at) {
        errno = EIO;
        return -1;
    }
    if (mode == Mode::interrupt_once && !interrupted) {
        interrupted = true;
        errno = EINTR;
        return -1;
    }
    if (mode == Mode::short_reads && n > 7)
        n = 7;
    return __real_pread(fd, buf, n, offset);
}

int main(int argc, char** argv) {
    CHECK(argc == 8);
    const char *gguf_dir = argv[1], *tensor = argv[2], *shard_dir = argv[4], *shard_name = argv[5],
               *prefix = argv[6];
    const std::vector<char> gguf_rows = slurp(argv[3]), mxfp4_rows = slurp(argv[7]);

    // GGUF: what a healthy, a short-reading and an interrupted file give.
    for (Mode m : {Mode::pass, Mode::short_reads, Mode::interrupt_once}) {
        set(m);
        kb200_gguf* g = nullptr;
        CHECK(kb200_gguf_open(gguf_dir, nullptr, &g) == KB200_OK);
        std::vector<char> got(gguf_rows.size());
        CHECK(kb200_gguf_read_packed_rows(g, tensor, 0, 0, got.data(), got.size(), nullptr) == KB200_OK);
        CHECK(got == gguf_rows);
        if (m == Mode::short_reads)
            CHECK(calls > long(gguf_rows.size() / 7));
        kb200_gguf_close(g);
    }
    // GGUF: an I/O error at each read in turn.
    long open_failures = 0, read_failures = 0;
    for (long k = 0;; ++k) {
        set(Mode::fail_at, k);
        kb200_gguf* g = nullptr;
        const int s = kb200_gguf_open(gguf_dir, nullptr, &g);
        if (s != KB200_OK) {
            CHECK(s == KB200_IO && std::strcmp(kb200::last_error, "gguf_read_failed") == 0 && g == nullptr);
            ++open_failures;
            continue;
        }
        std::vector<char> got(gguf_rows.size());
        const int r = kb200_gguf_read_packed_rows(g, tensor, 0, 0, got.data(), got.size(), nullptr);
        kb200_gguf_close(g);
        if (r != KB200_OK) {
            CHECK(r == KB200_IO && std::strcmp(kb200::last_error, "gguf_read_failed") == 0);
            ++read_failures;
            continue;
        }
        CHECK(got == gguf_rows);  // the injected failure came after every read
        break;
    }
    CHECK(open_failures > 0 && read_failures > 0);

    // Safetensors shard: the same three read behaviours, then failures.
    for (Mode m : {Mode::pass, Mode::short_reads, Mode::interrupt_once}) {
        set(m);
        kb200_shard* sh = nullptr;
        CHECK(kb200_shard_open(shard_dir, shard_name, nullptr, &sh) == KB200_OK);
        kb200_shard_tensor info{};
        CHECK(kb200_shard_find_tensor(sh, (std::string(prefix) + "_blocks").c_str(), &info) == KB200_OK);
        const uint64_t rows = info.shape[1], groups = info.shape[2];
        std::vector<char> w(rows * groups * 16), sc(rows * groups);
        uint64_t columns = 0;
        CHECK(kb200_shard_load_mxfp4_expert_rows(sh, prefix, 0, 0, rows, 1ull << 40, w.data(), w.size(), sc.data(),
                                                 sc.size(), &columns) == KB200_OK);
        std::vector<char> both(w);
        both.insert(both.end(), sc.begin(), sc.end());
        CHECK(both == mxfp4_rows && columns == groups * 32);
        kb200_shard_close(sh);
    }
    open_failures = read_failures = 0;
    for (long k = 0;; ++k) {
        set(Mode::fail_at, k);
        kb200_shard* sh = nullptr;
        const int s = kb200_shard_open(shard_dir, shard_name, nullptr, &sh);
        if (s != KB200_OK) {
            CHECK(s == KB200_IO && std::strcmp(kb200::last_error, "short_or_failed_read") == 0 && sh == nullptr);
            ++open_failures;
            continue;
        }
        kb200_shard_tensor info{};
        CHECK(kb200_shard_find_tensor(sh, (std::string(prefix) + "_blocks").c_str(), &info) == KB200_OK);
        const uint64_t rows = info.shape[1], groups = info.shape[2];
        std::vector<char> w(rows * groups * 16), sc(rows * groups);
        uint64_t columns = 0;
        const int r = kb200_shard_load_mxfp4_expert_rows(sh, prefix, 0, 0, rows, 1ull << 40, w.data(), w.size(),
                                                         sc.data(), sc.size(), &columns);
        kb200_shard_close(sh);
        if (r != KB200_OK) {
            CHECK(r == KB200_IO && std::strcmp(kb200::last_error, "short_or_failed_read") == 0);
            ++read_failures;
            continue;
        }
        break;
    }
    CHECK(open_failures > 0 && read_failures > 0);
    std::printf("ok\n");
    return 0;
}

// Opens every given checkpoint with the native readers and reads whatever the
// open reports, for memory-safety runs under AddressSanitizer and
// UndefinedBehaviorSanitizer: arguments are "gguf:<dir>" or
// "shard:<dir>/<name>". Failures to open are expected (malformed inputs); the
// run only has to finish. Prints the number of inputs opened and "ok".
#include <cstdio>
#include <cstring>
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

int main(int argc, char** argv) {
    int opened = 0;
    for (int i = 1; i < argc; ++i) {
        const std::string arg = argv[i];
        if (arg.rfind("gguf:", 0) == 0) {
            kb200_gguf* g = nullptr;
            if (kb200_gguf_open(arg.c_str() + 5, nullptr, &g) != KB200_OK)
                continue;
            ++opened;
            for (size_t t = 0; t < kb200_gguf_tensor_count(g); ++t) {
                kb200_gguf_tensor info{};
                const char* name = nullptr;
                if (kb200_gguf_tensor_at(g, t, &info, &name) != KB200_OK || info.rank < 2)
                    continue;
                std::vector<char> rows(info.row_bytes * info.shape[1]);
                kb200_gguf_read_packed_rows(g, name, 0, 0, rows.data(), rows.size(), nullptr);
                kb200_weight_identity id{};
                kb200_gguf_identity(g, name, info.shape[2] - 1, &id);
            }
            uint64_t v = 0;
            kb200_gguf_integer(g, "general.alignment", &v);
            kb200_gguf_close(g);
        } else if (arg.rfind("shard:", 0) == 0) {
            const std::string path = arg.substr(6);
            const size_t slash = path.rfind('/');
            kb200_shard* s = nullptr;
            if (kb200_shard_open(path.substr(0, slash).c_str(), path.substr(slash + 1).c_str(), nullptr, &s)
                != KB200_OK)
                continue;
            ++opened;
            for (size_t t = 0; t < kb200_shard_tensor_count(s); ++t) {
                kb200_shard_tensor info{};
                const char* name = nullptr;
                if (kb200_shard_tensor_at(s, t, &info, &name) != KB200_OK)
                    continue;
                std::vector<char> bytes(info.bytes + 1);
                kb200_shard_read_tensor(s, name, 0, bytes.data(), info.bytes);
                const size_t n = std::strlen(name);
                if (n > 7 && std::strcmp(name + n - 7, "_blocks") == 0 && info.rank == 4) {
                    const std::string prefix(name, n - 7);
                    std::vector<char> w(info.shape[1] * info.shape[2] * 16), sc(info.shape[1] * info.shape[2]);
                    uint64_t cols = 0;
                    kb200_shard_load_mxfp4_expert_rows(s, prefix.c_str(), 0, 0, info.shape[1], 1ull << 40, w.data(),
                                                       w.size(), sc.data(), sc.size(), &cols);
                }
            }
            kb200_shard_close(s);
        }
    }
    std::printf("%d ok\n", opened);
    return 0;
}

// Unit test of the source-read team (kadan_b200/csrc/read_team.hpp): row
// splitting follows the reference read team's boundaries, every item of a
// round runs exactly once whatever the lane count, rounds can follow one
// another and be empty, and the first failing item's status is reported
// after all items ran. Prints "ok" on success; exits non-zero otherwise.
#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <thread>
#include <vector>

#include "read_team.hpp"

using kb200::ReadItem;
using kb200::ReadTeam;
using kb200::split_read;

#define CHECK(c)                                                              \
    do {                                                                      \
        if (!(c)) {                                                           \
            std::fprintf(stderr, "%s:%d: check failed: %s\n", __FILE__, __LINE__, #c); \
            std::exit(1);                                                     \
        }                                                                     \
    } while (0)

namespace {

struct Counter {
    std::vector<std::atomic<int>> hits;
    explicit Counter(size_t n) : hits(n) {
        for (auto& h : hits)
            h = 0;
    }
};

// A source that fills each row with its row index and counts its calls per row.
int fill_rows(void* user, uint64_t first_row, void* dst, uint64_t bytes) {
    auto* c = static_cast<Counter*>(user);
    const uint64_t row_bytes = 1024;
    auto* out = static_cast<uint8_t*>(dst);
    for (uint64_t r = 0; r < bytes / row_bytes; ++r) {
        for (uint64_t b = 0; b < row_bytes; ++b)
            out[r * row_bytes + b] = uint8_t(first_row + r);
        c->hits[first_row + r].fetch_add(1);
    }
    return KB200_OK;
}

int failing(void* user, uint64_t first_row, void*, uint64_t) {
    static_cast<std::atomic<int>*>(user)->fetch_add(1);
    return first_row == 3 ? KB200_IO : KB200_OK;
}

}  // namespace

int main() {
    // Boundaries: rows / lanes * lane + rows % lanes * lane / lanes.
    for (int lanes : {1, 2, 3, 4, 7, 16}) {
        for (uint64_t rows : {1u, 3u, 4u, 5u, 2048u, 2049u, 4093u}) {
            std::vector<ReadItem> items;
            uint8_t* base = reinterpret_cast<uint8_t*>(uintptr_t(4096));
            split_read(items, fill_rows, nullptr, 100, rows, 1024, base, lanes);
            const bool whole = lanes <= 1 || rows * 1024 < kb200::kParallelReadBytes || rows < 4;
            if (whole) {
                CHECK(items.size() == 1 && items[0].first_row == 100 && items[0].bytes == rows * 1024);
                continue;
            }
            uint64_t next = 100;
            for (size_t i = 0; i < items.size(); ++i) {
                CHECK(items[i].first_row == next && items[i].bytes % 1024 == 0 && items[i].bytes > 0);
                CHECK(items[i].dst == base + (next - 100) * 1024);
                next += items[i].bytes / 1024;
            }
            CHECK(next == 100 + rows);
            CHECK(items.size() <= size_t(lanes));
        }
    }
    // Exactly once per row, over many rounds and lane counts.
    for (int lanes : {1, 2, 4, 8}) {
        ReadTeam team(lanes);
        CHECK(team.lanes() == lanes);
        for (int round = 0; round < 60; ++round) {
            const uint64_t rows = uint64_t(round * 37 % 3000);
            Counter c(rows ? rows : 1);
            std::vector<uint8_t> buffer(rows * 1024 + 1);
            std::vector<ReadItem> items;
            // Mixed items: one large tile split into runs, then small whole tiles.
            const uint64_t big = rows / 2;
            if (big)
                split_read(items, fill_rows, &c, 0, big, 1024, buffer.data(), lanes);
            for (uint64_t r = big; r < rows; r += 7) {
                const uint64_t n = std::min<uint64_t>(7, rows - r);
                split_read(items, fill_rows, &c, r, n, 1024, buffer.data() + r * 1024, lanes);
            }
            CHECK(team.run(items) == KB200_OK);
            for (uint64_t r = 0; r < rows; ++r) {
                CHECK(c.hits[r].load() == 1);
                CHECK(buffer[r * 1024] == uint8_t(r) && buffer[r * 1024 + 1023] == uint8_t(r));
            }
        }
        CHECK(team.run({}) == KB200_OK);
    }
    // A failing item: every item still runs, the failure is returned.
    {
        ReadTeam team(4);
        std::atomic<int> calls{0};
        std::vector<ReadItem> items;
        for (uint64_t i = 0; i < 9; ++i)
            items.push_back({failing, &calls, i, nullptr, 0});
        CHECK(team.run(items) == KB200_IO);
        CHECK(calls.load() == 9);
        calls = 0;
        items.resize(3);
        CHECK(team.run(items) == KB200_OK && calls.load() == 3);
    }
    // Teams come and go without leaving threads behind.
    for (int i = 0; i < 50; ++i) {
        ReadTeam team(1 + i % 6);
        Counter c(8);
        std::vector<uint8_t> buffer(8 * 1024);
        std::vector<ReadItem> items;
        split_read(items, fill_rows, &c, 0, 8, 1024, buffer.data(), 1);
        CHECK(team.run(items) == KB200_OK && c.hits[7].load() == 1);
    }
    std::printf("ok\n");
    return 0;
}

// Host read team for packed-row sources: the reference's PackedReadTeam
// (services/hikari/inference_worker/include/kadan/packed_read_team.hpp:22-275).
// Persistent worker threads and the calling thread drain one list of source
// reads; every item runs exactly once, and the first failure is reported after
// all lanes are done, so no source call is still running when run() returns.
#pragma once

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <mutex>
#include <thread>
#include <vector>

#include "kadan_b200.h"

namespace kb200 {

// One source call: `bytes` bytes of whole rows from `first_row` into `dst`.
struct ReadItem {
    kb200_row_source source;
    void* user;
    uint64_t first_row;
    uint8_t* dst;
    uint64_t bytes;
};

// A tile of at least this many bytes and four rows is read by all lanes,
// each taking a contiguous run of rows (packed_read_team.hpp:27, :87).
constexpr uint64_t kParallelReadBytes = 2ull * 1024 * 1024;

// Append the reads of `rows` rows of `row_bytes` from `first_row` into `dst`:
// one item, or `lanes` contiguous row runs with the reference's boundaries
// (rows / lanes * lane + rows % lanes * lane / lanes).
inline void split_read(std::vector<ReadItem>& items, kb200_row_source source, void* user, uint64_t first_row,
                       uint64_t rows, uint64_t row_bytes, uint8_t* dst, int lanes) {
    const uint64_t bytes = rows * row_bytes;
    if (lanes <= 1 || bytes < kParallelReadBytes || rows < 4) {
        items.push_back({source, user, first_row, dst, bytes});
        return;
    }
    const uint64_t n = uint64_t(lanes);
    auto boundary = [&](uint64_t lane) { return rows / n * lane + rows % n * lane / n; };
    for (uint64_t lane = 0; lane < n; ++lane) {
        const uint64_t a = boundary(lane), b = boundary(lane + 1);
        if (b > a)
            items.push_back({source, user, first_row + a, dst + a * row_bytes, (b - a) * row_bytes});
    }
}

class ReadTeam {
public:
    // Throws what std::thread throws when a worker cannot start; the workers
    // already started are joined first.
    explicit ReadTeam(int lanes) : lanes_(lanes < 1 ? 1 : lanes) {
        try {
            for (int w = 1; w < lanes_; ++w)
                workers_.emplace_back([this] { work(); });
        } catch (...) {
            stop();
            throw;
        }
    }
    ~ReadTeam() {
        stop();
    }
    ReadTeam(const ReadTeam&) = delete;
    ReadTeam& operator=(const ReadTeam&) = delete;

    int lanes() const {
        return lanes_;
    }

    // Runs every item; returns KB200_OK or the status of the first item that failed.
    int run(const std::vector<ReadItem>& items) {
        if (items.empty())
            return KB200_OK;
        {
            std::lock_guard<std::mutex> lock(mutex_);
            items_ = &items;
            next_.store(0);
            status_.store(KB200_OK);
            remaining_ = int(workers_.size());
            ++round_;
        }
        ready_.notify_all();
        drain();
        std::unique_lock<std::mutex> lock(mutex_);
        done_.wait(lock, [&] { return remaining_ == 0; });
        items_ = nullptr;
        return status_.load();
    }

private:
    void stop() {
        {
            std::lock_guard<std::mutex> lock(mutex_);
            stopping_ = true;
        }
        ready_.notify_all();
        for (auto& t : workers_)
            if (t.joinable())
                t.join();
    }

    void drain() {
        const auto& items = *items_;
        for (size_t i; (i = next_.fetch_add(1)) < items.size();) {
            const ReadItem& it = items[i];
            const int s = it.source(it.user, it.first_row, it.dst, it.bytes);
            if (s != KB200_OK) {
                int ok = KB200_OK;
                status_.compare_exchange_strong(ok, s);
            }
        }
    }

    void work() {
        uint64_t seen = 0;
        for (;;) {
            {
                std::unique_lock<std::mutex> lock(mutex_);
                ready_.wait(lock, [&] { return stopping_ || round_ != seen; });
                if (stopping_)
                    return;
                seen = round_;
            }
            drain();
            {
                std::lock_guard<std::mutex> lock(mutex_);
                --remaining_;
            }
            done_.notify_all();
        }
    }

    const int lanes_;
    std::vector<std::thread> workers_;
    std::mutex mutex_;
    std::condition_variable ready_, done_;
    const std::vector<ReadItem>* items_ = nullptr;
    std::atomic<size_t> next_{0};
    std::atomic<int> status_{KB200_OK};
    int remaining_ = 0;
    uint64_t round_ = 0;
    bool stopping_ = false;
};

}  // namespace kb200

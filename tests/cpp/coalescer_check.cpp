// coalescer_check.cpp — host-only test of fe::Coalescer (fastembed_b200/csrc/host/coalescer.h),
// the merging of concurrent SentenceTransformer calls into one device batch.
//
// Threads submit requests of 1-5 items to a batch function that doubles each item and
// takes a little time, as a device pass would.  Checks: every caller gets exactly its own
// results, in order; merged batches happen under contention; no batch of several calls
// exceeds the item cap; a batch function that throws fails every call of that batch and
// no other; with the cap at 0 no calls merge.  Prints "ok" and exits 0 on success.
#include <atomic>
#include <chrono>
#include <cstdio>
#include <stdexcept>
#include <thread>
#include <vector>

#include "coalescer.h"

namespace {

int failures = 0;

void expect(bool ok, const char *what)
{
    if (!ok) {
        std::fprintf(stderr, "FAILED: %s\n", what);
        ++failures;
    }
}

struct Run {
    std::atomic<int> max_batch_items{0};
    std::atomic<int> batches{0};
};

void stress(size_t cap, int threads, int calls, bool poison, Run &run, std::atomic<int> &mismatches,
            std::atomic<int> &poison_ok, std::atomic<int> &poison_bad)
{
    fe::Coalescer<int, long> co(
        [&](const std::vector<int> &items) {
            run.batches++;
            int n = static_cast<int>(items.size());
            int prev = run.max_batch_items.load();
            while (n > prev && !run.max_batch_items.compare_exchange_weak(prev, n)) {
            }
            std::this_thread::sleep_for(std::chrono::microseconds(300));
            std::vector<long> out;
            for (int v : items) {
                if (v < 0) throw std::runtime_error("poisoned batch");
                out.push_back(2L * v);
            }
            return out;
        },
        cap);
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t)
        pool.emplace_back([&, t] {
            for (int c = 0; c < calls; ++c) {
                const int k = 1 + (t * 7 + c * 3) % 5;
                std::vector<int> items;
                for (int i = 0; i < k; ++i) items.push_back(t * 100000 + c * 10 + i);
                const bool bad = poison && c % 17 == 5 && t % 3 == 0;
                if (bad) items[k / 2] = -1;
                try {
                    std::vector<long> got = co.submit(items);
                    if (bad) {
                        poison_bad++;  // a poisoned call must fail
                        continue;
                    }
                    bool same = got.size() == items.size();
                    for (size_t i = 0; same && i < items.size(); ++i) same = got[i] == 2L * items[i];
                    if (!same) mismatches++;
                } catch (const std::runtime_error &) {
                    if (bad) poison_ok++;
                    // an innocent call may share a poisoned batch; it must then fail too, which is
                    // what the batch's exception means, so nothing to count here
                }
            }
        });
    for (auto &th : pool) th.join();
    const auto st = co.stats();
    expect(st.calls == static_cast<uint64_t>(threads) * calls, "every call is served exactly once");
    if (cap > 0 && threads > 1) expect(st.max_calls_in_batch > 1, "concurrent calls are merged");
    if (cap == 0) expect(st.max_calls_in_batch == 1, "cap 0 never merges");
}

}  // namespace

int main()
{
    {
        Run run;
        std::atomic<int> mism{0}, pok{0}, pbad{0};
        stress(64, 16, 60, false, run, mism, pok, pbad);
        expect(mism.load() == 0, "each caller gets its own results in order");
        expect(run.max_batch_items.load() <= 64, "a merged batch stays within the item cap");
    }
    {
        Run run;
        std::atomic<int> mism{0}, pok{0}, pbad{0};
        stress(64, 12, 60, true, run, mism, pok, pbad);
        expect(mism.load() == 0, "results stay correct around poisoned batches");
        expect(pbad.load() == 0, "a poisoned call never returns results");
        expect(pok.load() > 0, "poisoned calls raise the batch's exception");
    }
    {
        Run run;
        std::atomic<int> mism{0}, pok{0}, pbad{0};
        stress(0, 8, 30, false, run, mism, pok, pbad);
        expect(mism.load() == 0, "unmerged calls get their own results");
        expect(run.max_batch_items.load() <= 5, "cap 0 runs one call per batch");
    }
    {
        // a single request larger than the cap still runs (alone)
        fe::Coalescer<int, int> co([](const std::vector<int> &v) { return v; }, 4);
        std::vector<int> big(10, 7);
        expect(co.submit(big) == big, "an oversize request runs alone");
        expect(co.submit(std::vector<int>{}).empty(), "an empty request returns nothing");
    }
    {
        // a batch function returning the wrong count is reported to the caller
        fe::Coalescer<int, int> co([](const std::vector<int> &) { return std::vector<int>{1}; }, 4);
        bool threw = false;
        try {
            (void)co.submit(std::vector<int>{1, 2});
        } catch (const std::logic_error &) {
            threw = true;
        }
        expect(threw, "a short result list raises");
    }
    if (failures) return 1;
    std::printf("ok\n");
    return 0;
}

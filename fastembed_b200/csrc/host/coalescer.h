// coalescer.h — merges concurrent encode calls into one device batch.
//
// The reference's HTTP server shares one model object between its worker threads
// (http_server.cpp:136, :177) and encodes each request on its own, so concurrent
// requests each run a whole forward pass over a handful of tokens.  A Coalescer gives
// that call pattern one packed pass per group of concurrent calls ("natural batching"):
//   - submit() queues the caller's items and blocks until its results are ready;
//   - while a batch runs, later callers wait in the queue;
//   - when no batch is running, one waiting caller becomes the leader: it takes the
//     queued requests in arrival order, up to `max_items` items in total (always at
//     least one request), runs them as one batch through the batch function and hands
//     each caller its own results.
// There is no timer: a caller that finds nothing running starts at once, so an idle
// server adds no latency, and a busy one batches whatever arrived meanwhile.
// The batch function returns one result per item, in input order.  If it throws,
// every caller in that batch gets the exception; input errors that concern a single
// caller are to be checked before submit(), in the caller's own thread.
#pragma once

#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <deque>
#include <exception>
#include <functional>
#include <mutex>
#include <stdexcept>
#include <utility>
#include <vector>

namespace fe {

template <class Item, class Result>
class Coalescer {
public:
    using BatchFn = std::function<std::vector<Result>(const std::vector<Item> &)>;

    struct Stats {
        uint64_t calls = 0;    // submit() calls served
        uint64_t batches = 0;  // batch-function runs
        uint64_t items = 0;    // items run
        uint64_t max_calls_in_batch = 0;
    };

    // max_items == 0: no merging, one call per batch.
    Coalescer(BatchFn fn, size_t max_items) : fn_(std::move(fn)), max_items_(max_items) {}

    std::vector<Result> submit(const std::vector<Item> &items)
    {
        Req req;
        req.items = &items;
        std::unique_lock<std::mutex> lk(mu_);
        queue_.push_back(&req);
        while (!req.done) {
            if (busy_) {
                cv_.wait(lk);
                continue;
            }
            busy_ = true;
            std::vector<Req *> group;
            size_t n = 0;
            while (!queue_.empty()) {
                Req *r = queue_.front();
                const size_t k = r->items->size();
                if (!group.empty() && (max_items_ == 0 || n + k > max_items_)) break;
                group.push_back(r);
                queue_.pop_front();
                n += k;
            }
            lk.unlock();
            run_group(group, n);
            lk.lock();
            for (Req *r : group) r->done = true;
            stats_.calls += group.size();
            stats_.batches += 1;
            stats_.items += n;
            if (group.size() > stats_.max_calls_in_batch) stats_.max_calls_in_batch = group.size();
            busy_ = false;
            cv_.notify_all();
        }
        lk.unlock();
        if (req.err) std::rethrow_exception(req.err);
        return std::move(req.out);
    }

    Stats stats() const
    {
        std::lock_guard<std::mutex> lk(mu_);
        return stats_;
    }

private:
    struct Req {
        const std::vector<Item> *items = nullptr;
        std::vector<Result> out;
        std::exception_ptr err;
        bool done = false;
    };

    // Runs outside the lock; writes only the requests of `group`, which no other
    // thread touches until they are marked done.
    void run_group(const std::vector<Req *> &group, size_t n)
    {
        try {
            if (group.size() == 1) {
                group[0]->out = fn_(*group[0]->items);
                if (group[0]->out.size() != group[0]->items->size())
                    throw std::logic_error("coalescer: batch function returned the wrong number of results");
                return;
            }
            std::vector<Item> all;
            all.reserve(n);
            for (Req *r : group) all.insert(all.end(), r->items->begin(), r->items->end());
            std::vector<Result> res = fn_(all);
            if (res.size() != all.size())
                throw std::logic_error("coalescer: batch function returned the wrong number of results");
            size_t off = 0;
            for (Req *r : group) {
                const size_t k = r->items->size();
                r->out.assign(std::make_move_iterator(res.begin() + off), std::make_move_iterator(res.begin() + off + k));
                off += k;
            }
        } catch (...) {
            const std::exception_ptr e = std::current_exception();
            for (Req *r : group) {
                r->out.clear();
                r->err = e;
            }
        }
    }

    BatchFn fn_;
    size_t max_items_;
    mutable std::mutex mu_;
    std::condition_variable cv_;
    std::deque<Req *> queue_;
    bool busy_ = false;
    Stats stats_;
};

}  // namespace fe

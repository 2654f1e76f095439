#include "router.hpp"

#include <algorithm>
#include <unordered_set>

#include <cuda_runtime.h>

#include <limits>

namespace nvllm {

void TokenStream::push(const TokenEvent& ev) {
    {
        std::lock_guard<std::mutex> lk(mu_);
        if (closed_) return;
        q_.push_back(ev);
        if (ev.finished) closed_ = true;
    }
    cv_.notify_all();
}

std::optional<TokenEvent> TokenStream::pop_wait() {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [&] { return !q_.empty() || closed_; });
    if (q_.empty()) return std::nullopt;
    TokenEvent ev = q_.front();
    q_.pop_front();
    return ev;
}

std::optional<TokenEvent> TokenStream::pop_wait_for(std::chrono::milliseconds timeout) {
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait_for(lk, timeout, [&] { return !q_.empty() || closed_; });
    if (q_.empty()) return std::nullopt;
    TokenEvent ev = q_.front();
    q_.pop_front();
    return ev;
}

void TokenStream::close() {
    {
        std::lock_guard<std::mutex> lk(mu_);
        closed_ = true;
    }
    cv_.notify_all();
}

bool TokenStream::closed() const {
    std::lock_guard<std::mutex> lk(mu_);
    return closed_;
}

Router::Router(std::span<Generator* const> gens) {
    lanes_.reserve(gens.size());
    for (Generator* g : gens) {
        auto lane = std::make_unique<Lane>();
        lane->gen = g;
        lane->snapshot = g->metrics();
        lanes_.push_back(std::move(lane));
    }
    for (auto& lane : lanes_) {
        Lane& l = *lane;
        l.thread = std::jthread([this, &l](std::stop_token st) { engine_loop(st, l); });
    }
}

Router::~Router() {
    for (auto& lane : lanes_) {
        lane->thread.request_stop();
        lane->cv.notify_all();
    }
    for (auto& lane : lanes_) {
        if (lane->thread.joinable()) lane->thread.join();
    }
}

std::expected<int32_t, EngineError> Router::add_request(SeqId id, std::vector<int64_t> prompt,
                                                        std::size_t max_new_tokens,
                                                        std::shared_ptr<TokenStream> stream) {
    if (prompt.empty()) prompt.push_back(1);  // as Sequence does (src/scheduler.cpp:8-20)
    max_new_tokens = std::max<std::size_t>(max_new_tokens, 1);
    const uint64_t rows = prompt.size() + max_new_tokens;
    int32_t best = -1;
    {
        std::lock_guard<std::mutex> lk(route_mu_);
        if (owner_.contains(id)) return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
        uint64_t best_load = std::numeric_limits<uint64_t>::max();
        for (std::size_t i = 0; i < lanes_.size(); ++i) {
            const uint64_t l = lanes_[i]->load.load() + lanes_[i]->queued_rows.load();
            if (l < best_load) {
                best_load = l;
                best = int32_t(i);
            }
        }
        if (best < 0) return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
        owner_[id] = best;
        Lane& l = *lanes_[best];
        // counted before the request is visible to the thread, so a decision
        // taken right after this one sees it
        l.queued_rows += rows;
        l.placed += 1;
        {
            std::lock_guard<std::mutex> lq(l.mu);
            l.ingress.push_back(Pending{id, std::move(prompt), max_new_tokens, std::move(stream)});
            l.busy = true;
        }
        l.cv.notify_one();
    }
    return best;
}

std::expected<void, EngineError> Router::add_requests(std::span<const SeqId> ids,
                                                      std::span<std::vector<int64_t>> prompts,
                                                      std::span<const std::size_t> max_new,
                                                      std::span<int32_t> gpus) {
    const std::size_t n = ids.size();
    if (prompts.size() != n || max_new.size() != n || (!gpus.empty() && gpus.size() != n) ||
        lanes_.empty()) {
        return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    }
    std::vector<std::vector<Pending>> per_lane(lanes_.size());
    std::vector<uint64_t> rows_to(lanes_.size(), 0);
    {
        std::lock_guard<std::mutex> lk(route_mu_);
        std::unordered_set<SeqId> fresh;
        for (SeqId id : ids) {
            if (owner_.contains(id) || !fresh.insert(id).second) {
                return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
            }
        }
        std::vector<uint64_t> load(lanes_.size());
        for (std::size_t i = 0; i < lanes_.size(); ++i) {
            load[i] = lanes_[i]->load.load() + lanes_[i]->queued_rows.load();
        }
        for (std::size_t k = 0; k < n; ++k) {
            std::vector<int64_t>& prompt = prompts[k];
            if (prompt.empty()) prompt.push_back(1);  // as Sequence does (src/scheduler.cpp:8-20)
            const std::size_t mx = std::max<std::size_t>(max_new[k], 1);
            const uint64_t rows = prompt.size() + mx;
            const auto best = std::size_t(std::min_element(load.begin(), load.end()) - load.begin());
            load[best] += rows;
            rows_to[best] += rows;
            owner_[ids[k]] = int32_t(best);
            if (!gpus.empty()) gpus[k] = int32_t(best);
            per_lane[best].push_back(Pending{ids[k], std::move(prompt), mx, {}});
        }
        // counted before the requests are visible to the threads
        for (std::size_t i = 0; i < lanes_.size(); ++i) {
            if (per_lane[i].empty()) continue;
            lanes_[i]->queued_rows += rows_to[i];
            lanes_[i]->placed += per_lane[i].size();
        }
    }
    for (std::size_t i = 0; i < lanes_.size(); ++i) {
        if (per_lane[i].empty()) continue;
        Lane& l = *lanes_[i];
        {
            std::lock_guard<std::mutex> lq(l.mu);
            for (Pending& p : per_lane[i]) l.ingress.push_back(std::move(p));
            l.busy = true;
        }
        l.cv.notify_one();
    }
    return {};
}

void Router::signal_idle() {
    {
        std::lock_guard<std::mutex> li(idle_mu_);
        ++idle_events_;
    }
    idle_cv_.notify_all();
}

void Router::engine_loop(std::stop_token stop, Lane& l) {
    cudaSetDevice(l.gen->device());
    std::deque<Pending> batch;
    // tokens go to the streams of the requests that asked for them
    l.gen->set_token_sink([&l](const TokenEvent& ev) {
        auto it = l.streams.find(ev.seq_id);
        if (it == l.streams.end()) return;
        it->second->push(ev);
        if (ev.finished) l.streams.erase(it);
    });
    // no lock is held while idle_mu_ is taken (wait_idle takes the lanes'
    // locks while it holds none either)
    auto stop_with = [&](EngineError e) {
        for (auto& [id, st] : l.streams) st->close();
        l.streams.clear();
        {
            std::lock_guard<std::mutex> lk(l.mu);
            l.failed = true;
            l.error = e;
            l.busy = false;
            l.snapshot = l.gen->metrics();
        }
        signal_idle();
    };
    while (!stop.stop_requested()) {
        bool idle = false;
        {
            std::lock_guard<std::mutex> lk(l.mu);
            if (l.ingress.empty() && !l.gen->has_pending_work()) {
                l.busy = false;
                l.snapshot = l.gen->metrics();
                idle = true;
            } else {
                batch.swap(l.ingress);
            }
        }
        if (idle) {
            signal_idle();
            std::unique_lock<std::mutex> lk(l.mu);
            l.cv.wait(lk, stop, [&] { return !l.ingress.empty(); });
            if (stop.stop_requested()) break;
            batch.swap(l.ingress);
        }
        uint64_t moved = 0;
        for (Pending& p : batch) {
            moved += p.prompt.size() + p.max_new;
            if (p.stream) l.streams[p.id] = std::move(p.stream);
            l.gen->add_request(p.id, std::move(p.prompt), p.max_new);
        }
        batch.clear();
        // publish the new load before the queued rows leave the count, so the
        // router never sees this GPU lighter than it is
        l.load = l.gen->outstanding_tokens();
        l.queued_rows -= moved;
        if (!l.gen->has_pending_work()) continue;
        auto r = l.gen->step();
        if (!r) {
            stop_with(r.error());
            return;
        }
        if (r->batch_size == 0 && l.gen->has_pending_work()) {
            // the queue head can never be admitted (larger than the arena)
            stop_with(EngineError{EngineError::Kind::Invalid, 0});
            return;
        }
        l.load = l.gen->outstanding_tokens();
        {
            std::lock_guard<std::mutex> lk(l.mu);
            l.snapshot = l.gen->metrics();
        }
    }
    // stopped: no further tokens will come for the requests still held here
    for (auto& [id, st] : l.streams) st->close();
    l.streams.clear();
}

std::expected<void, EngineError> Router::wait_idle() {
    for (;;) {
        uint64_t seen;
        {
            std::lock_guard<std::mutex> li(idle_mu_);
            seen = idle_events_;
        }
        bool all_idle = true;
        for (auto& lane : lanes_) {
            std::lock_guard<std::mutex> lq(lane->mu);
            if (lane->failed) return std::unexpected(lane->error);
            if (lane->busy || !lane->ingress.empty()) all_idle = false;
        }
        if (all_idle) return {};
        std::unique_lock<std::mutex> li(idle_mu_);
        idle_cv_.wait_for(li, std::chrono::milliseconds(100),
                          [&] { return idle_events_ != seen; });
    }
}

std::optional<std::vector<int64_t>> Router::output(SeqId id) {
    int32_t gpu = -1;
    {
        std::lock_guard<std::mutex> lk(route_mu_);
        auto it = owner_.find(id);
        if (it == owner_.end()) return std::nullopt;
        gpu = it->second;
    }
    Lane& l = *lanes_[gpu];
    // While the lane is idle its thread waits for l.mu before it touches the
    // generator again, so the generator is read here under that lock only.
    std::lock_guard<std::mutex> lk(l.mu);
    if (l.busy) return std::nullopt;
    const std::vector<int64_t>* t = l.gen->output(id);
    if (t == nullptr) return std::nullopt;
    return *t;
}

Metrics Router::metrics(int32_t gpu) {
    if (gpu < 0 || gpu >= num_gpus()) return Metrics{};
    Lane& l = *lanes_[gpu];
    std::lock_guard<std::mutex> lk(l.mu);
    return l.snapshot;
}

uint64_t Router::placed(int32_t gpu) const noexcept {
    if (gpu < 0 || gpu >= int32_t(lanes_.size())) return 0;
    return lanes_[gpu]->placed.load();
}

}  // namespace nvllm

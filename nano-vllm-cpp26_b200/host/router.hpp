// Router: one request stream over the GPUs of a box, sequence-partitioned.
//
// The reference runs one ContinuousBatchingEngine: an ingress queue filled by
// the server thread (src/engine.cpp:89-104) and one engine thread
// (std::jthread, :79-81) that runs schedule -> forward_batch -> process
// outputs (:163-246). Here each GPU has its own Generator (its own arena,
// block allocator, scheduler and device model) and its own engine thread with
// its own ingress queue, and the router places every incoming request on the
// GPU with the least outstanding work: the rows still to run through the
// forward pass (uncomputed prompt tokens + tokens still to generate) of what
// that GPU holds or has queued. There is no collective: the GPUs share
// nothing but the router's bookkeeping.
//
// Threading: add_request, wait_idle, output and metrics may be called from
// any thread; each Generator is touched only by its own engine thread once the
// router owns it.
#pragma once

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <expected>
#include <memory>
#include <mutex>
#include <optional>
#include <span>
#include <thread>
#include <unordered_map>
#include <vector>

#include "generator.hpp"

namespace nvllm {

// Thread-safe channel of one request's tokens, from its GPU's engine thread to
// a client (the reference's TokenStreamQueue, include/nano_vllm/scheduler.hpp:
// 33-74): closed by the sequence's last token, or by the client going away.
class TokenStream {
public:
    void push(const TokenEvent& ev);
    // The next event; empty once the stream is closed and drained.
    std::optional<TokenEvent> pop_wait();
    // As pop_wait, giving up after `timeout` (empty; check closed()).
    std::optional<TokenEvent> pop_wait_for(std::chrono::milliseconds timeout);
    void close();
    bool closed() const;

private:
    mutable std::mutex mu_;
    std::condition_variable cv_;
    std::deque<TokenEvent> q_;
    bool closed_ = false;
};

class Router {
public:
    // gens[i] drives GPU gens[i]->device(); the router starts one engine
    // thread per generator. The generators must outlive the router.
    explicit Router(std::span<Generator* const> gens);
    ~Router();  // stops and joins the engine threads (pending work is dropped)
    Router(const Router&) = delete;
    Router& operator=(const Router&) = delete;

    // Places the request on the least-loaded GPU; returns that GPU's index in
    // gens, or an error when seq_id is already in use.
    std::expected<int32_t, EngineError> add_request(SeqId id, std::vector<int64_t> prompt,
                                                    std::size_t max_new_tokens,
                                                    std::shared_ptr<TokenStream> stream = {});
    // Places a burst of requests in one decision pass (each on the GPU that is
    // least loaded counting the ones placed before it in the burst), then
    // wakes each GPU once: its engine thread finds its whole share queued
    // instead of ingesting it over many small iterations. All or nothing:
    // a seq_id already in use, or repeated in the burst, places none. gpus
    // (when given) receives each request's GPU.
    std::expected<void, EngineError> add_requests(std::span<const SeqId> ids,
                                                  std::span<std::vector<int64_t>> prompts,
                                                  std::span<const std::size_t> max_new,
                                                  std::span<int32_t> gpus = {});
    // Blocks until every GPU is idle with an empty ingress queue (or one has
    // failed: its error is returned).
    std::expected<void, EngineError> wait_idle();
    // The finished token list of a request; empty while its GPU is busy or when
    // the request is unknown or unfinished.
    std::optional<std::vector<int64_t>> output(SeqId id);
    // Per-GPU telemetry, taken by each engine thread after every step.
    Metrics metrics(int32_t gpu);
    int32_t num_gpus() const noexcept { return int32_t(lanes_.size()); }
    // Requests placed on each GPU so far.
    uint64_t placed(int32_t gpu) const noexcept;

private:
    struct Pending {
        SeqId id;
        std::vector<int64_t> prompt;
        std::size_t max_new;
        std::shared_ptr<TokenStream> stream;
    };
    struct Lane {
        Generator* gen = nullptr;
        std::mutex mu;
        std::condition_variable_any cv;  // woken by a request or a stop request
        std::deque<Pending> ingress;          // guarded by mu
        std::atomic<uint64_t> load{0};        // outstanding rows published by the thread
        std::atomic<uint64_t> queued_rows{0};  // rows waiting in ingress
        std::atomic<bool> busy{false};        // ingress non-empty or work pending
        std::atomic<uint64_t> placed{0};
        Metrics snapshot;                      // guarded by mu, refreshed every step
        // streams of the requests on this GPU (engine thread only)
        std::unordered_map<SeqId, std::shared_ptr<TokenStream>> streams;
        EngineError error{};
        bool failed = false;                   // guarded by mu
        std::jthread thread;
    };
    void engine_loop(std::stop_token stop, Lane& lane);
    void signal_idle();

    std::vector<std::unique_ptr<Lane>> lanes_;
    std::mutex route_mu_;                      // placement decisions and owner_
    std::unordered_map<SeqId, int32_t> owner_;
    std::mutex idle_mu_;
    std::condition_variable idle_cv_;
    uint64_t idle_events_ = 0;  // guarded by idle_mu_: lanes that went idle or failed
};

}  // namespace nvllm

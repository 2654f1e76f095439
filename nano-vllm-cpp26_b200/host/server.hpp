// HttpServer: the reference's HTTP/SSE front end (HttpSseServer,
// src/server.cpp:114-209) in front of the device engine: the same three
// routes and wire format, with requests served by a Router over the box's
// GPUs instead of one CPU engine.
//
//   GET  /health       -> 200 "OK"
//   GET  /v1/metrics   -> the MetricsSnapshot JSON (src/engine.cpp:8-38) summed
//                         over the GPUs, plus "gpus": one snapshot per GPU
//   POST /v1/generate  {"prompt": "...", "max_tokens": n} -> text/event-stream,
//                      one frame per generated token:
//                      data: {"seq_id":S,"token_id":T,"text":"...","finished":B[,"ttft_us":U]}
//
// Prompts are tokenised as the reference's engine does (tokenize_prompt,
// src/engine.cpp:40-64) and token ids rendered as the reference model's
// vocabulary strings (src/model.cpp:114-121), so that the same model and
// prompt give the same frames. One thread accepts; each client gets its own
// thread, which waits on its request's TokenStream.
#pragma once

#include <atomic>
#include <cstdint>
#include <expected>
#include <memory>
#include <mutex>
#include <string>
#include <string_view>
#include <thread>
#include <vector>

#include "router.hpp"

namespace nvllm {

// The reference engine's whitespace-split djb2 word hashing (src/engine.cpp:40-64).
std::vector<int64_t> tokenize_prompt(std::string_view prompt, std::size_t vocab_size);
// The reference model's vocabulary string of a token id (src/model.cpp:114-121).
std::string token_text(int64_t token);

struct ServerConfig {
    std::string bind_address = "127.0.0.1";
    uint16_t port = 0;  // 0: any free port (see HttpServer::port)
    std::size_t vocab_size = 0;
};

class HttpServer {
public:
    // Binds and starts accepting on a background thread.
    static std::expected<std::unique_ptr<HttpServer>, EngineError> start(Router& router,
                                                                         const ServerConfig& cfg);
    // Stops accepting, closes the open streams and joins every thread.
    ~HttpServer();
    HttpServer(const HttpServer&) = delete;
    HttpServer& operator=(const HttpServer&) = delete;

    uint16_t port() const noexcept { return port_; }
    uint64_t requests_served() const noexcept { return served_.load(); }

private:
    HttpServer(Router& router, const ServerConfig& cfg) : router_(router), cfg_(cfg) {}
    void accept_loop(std::stop_token stop);
    void handle_client(int fd);
    std::string metrics_json();

    Router& router_;
    ServerConfig cfg_;
    int listen_fd_ = -1;
    uint16_t port_ = 0;
    std::atomic<uint64_t> next_seq_{1};
    std::atomic<uint64_t> served_{0};
    bool stopping_ = false;  // guarded by clients_mu_
    struct Client {
        std::shared_ptr<std::atomic<bool>> done;
        std::jthread thread;
    };
    std::mutex clients_mu_;
    std::vector<Client> clients_;
    std::vector<std::shared_ptr<TokenStream>> open_;  // guarded by clients_mu_
    std::jthread acceptor_;
};

}  // namespace nvllm

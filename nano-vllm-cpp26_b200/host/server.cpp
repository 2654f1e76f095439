#include "server.hpp"

#include <arpa/inet.h>
#include <netinet/in.h>
#include <poll.h>
#include <signal.h>
#include <sys/socket.h>
#include <unistd.h>

#include <array>
#include <charconv>
#include <chrono>
#include <condition_variable>
#include <format>

namespace nvllm {

namespace {

// The reference model's vocabulary words (src/model.cpp:114-116); token i reads
// as " " + word[i % 16] (src/model.cpp:118-121). Kept alike: it is the text of
// every streamed frame.
constexpr std::array<std::string_view, 16> kWords = {
    "system", "kernel", "cpp26", "batch",  "token",   "cache",      "paged",   "memory",
    "tensor", "matrix", "stream", "async", "latency", "throughput", "compute", "sched"};

bool is_space(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }

bool send_all(int fd, std::string_view data) {
    std::size_t sent = 0;
    while (sent < data.size()) {
        const ssize_t n = ::send(fd, data.data() + sent, data.size() - sent, MSG_NOSIGNAL);
        if (n <= 0) return false;
        sent += std::size_t(n);
    }
    return true;
}

// Position just past `"key"` and the colon after it, or npos.
std::size_t value_start(std::string_view body, std::string_view key) {
    const std::string quoted = std::format("\"{}\"", key);
    std::size_t pos = body.find(quoted);
    if (pos == std::string_view::npos) return pos;
    pos = body.find(':', pos + quoted.size());
    if (pos == std::string_view::npos) return pos;
    ++pos;
    while (pos < body.size() && is_space(body[pos])) ++pos;
    return pos;
}

// A JSON string value (with \" \\ \n \t escapes), or the fallback.
std::string json_string(std::string_view body, std::string_view key, std::string_view fallback) {
    std::size_t pos = value_start(body, key);
    if (pos == std::string_view::npos || pos >= body.size() || body[pos] != '"') {
        return std::string(fallback);
    }
    std::string out;
    for (++pos; pos < body.size(); ++pos) {
        const char c = body[pos];
        if (c == '"') return out;
        if (c == '\\' && pos + 1 < body.size()) {
            const char e = body[++pos];
            out.push_back(e == 'n' ? '\n' : e == 't' ? '\t' : e == 'r' ? '\r' : e);
        } else {
            out.push_back(c);
        }
    }
    return std::string(fallback);  // unterminated
}

std::size_t json_usize(std::string_view body, std::string_view key, std::size_t fallback) {
    const std::size_t pos = value_start(body, key);
    if (pos == std::string_view::npos) return fallback;
    std::size_t v = fallback;
    std::from_chars(body.data() + pos, body.data() + body.size(), v);
    return v;
}

// Reads one request: headers, then Content-Length bytes of body (at most 1 MiB).
bool read_request(int fd, std::string& req, std::size_t& body_at) {
    constexpr std::size_t kMax = std::size_t(1) << 20;
    char buf[8192];
    body_at = std::string::npos;
    std::size_t need = 0;
    for (;;) {
        if (body_at == std::string::npos) {
            const std::size_t h = req.find("\r\n\r\n");
            if (h != std::string::npos) {
                body_at = h + 4;
                const std::size_t cl = req.find("Content-Length:");
                if (cl != std::string::npos && cl < h) {
                    std::size_t v = 0;
                    std::size_t p = cl + 15;
                    while (p < h && is_space(req[p])) ++p;
                    std::from_chars(req.data() + p, req.data() + h, v);
                    need = v;
                }
            }
        }
        if (body_at != std::string::npos && req.size() >= body_at + need) return true;
        if (req.size() > kMax) return false;
        const ssize_t n = ::recv(fd, buf, sizeof(buf), 0);
        if (n <= 0) return body_at != std::string::npos;
        req.append(buf, std::size_t(n));
    }
}

std::string gpu_json(int32_t gpu, const Metrics& m) {
    return std::format(
        "{{\"gpu\": {}, \"requests_completed\": {}, \"tokens_generated\": {}, "
        "\"active_batch_size\": {}, \"waiting_queue_depth\": {}, \"kv_cache_used_blocks\": {}, "
        "\"kv_cache_total_blocks\": {}, \"iterations\": {}, \"avg_iteration_latency_ms\": {:.3f}, "
        "\"tokens_computed\": {}, \"h2d_bytes\": {}, \"d2h_bytes\": {}, \"kernel_launches\": {}}}",
        gpu, m.total_requests_completed, m.total_tokens_generated, m.active_batch_size,
        m.waiting_queue_depth, m.kv_cache_used_blocks, m.kv_cache_total_blocks, m.total_iterations,
        m.avg_iteration_latency_ms, m.total_tokens_computed, m.h2d_bytes, m.d2h_bytes,
        m.kernel_launches);
}

}  // namespace

std::vector<int64_t> tokenize_prompt(std::string_view prompt, std::size_t vocab_size) {
    std::vector<int64_t> tokens;
    const uint64_t mod = vocab_size > 1 ? uint64_t(vocab_size - 1) : 1;
    std::size_t pos = 0;
    while (pos < prompt.size()) {
        while (pos < prompt.size() && is_space(prompt[pos])) ++pos;
        if (pos >= prompt.size()) break;
        uint64_t h = 5381;  // djb2 over the word's bytes
        while (pos < prompt.size() && !is_space(prompt[pos])) {
            h = h * 33 + static_cast<unsigned char>(prompt[pos]);
            ++pos;
        }
        tokens.push_back(int64_t(h % mod) + 1);
    }
    if (tokens.empty()) tokens.push_back(1);
    return tokens;
}

std::string token_text(int64_t token) {
    return std::string(" ") + std::string(kWords[std::size_t(token < 0 ? 0 : token) % 16]);
}

std::expected<std::unique_ptr<HttpServer>, EngineError> HttpServer::start(
    Router& router, const ServerConfig& cfg) {
    if (cfg.vocab_size < 2) return std::unexpected(EngineError{EngineError::Kind::Invalid, 0});
    ::signal(SIGPIPE, SIG_IGN);
    std::unique_ptr<HttpServer> s(new HttpServer(router, cfg));
    s->listen_fd_ = ::socket(AF_INET, SOCK_STREAM, 0);
    if (s->listen_fd_ < 0) return std::unexpected(EngineError{EngineError::Kind::Invalid, errno});
    int one = 1;
    ::setsockopt(s->listen_fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in addr{};
    addr.sin_family = AF_INET;
    addr.sin_port = htons(cfg.port);
    if (::inet_pton(AF_INET, cfg.bind_address.c_str(), &addr.sin_addr) != 1 ||
        ::bind(s->listen_fd_, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) < 0 ||
        ::listen(s->listen_fd_, 128) < 0) {
        return std::unexpected(EngineError{EngineError::Kind::Invalid, errno});
    }
    socklen_t len = sizeof(addr);
    ::getsockname(s->listen_fd_, reinterpret_cast<sockaddr*>(&addr), &len);
    s->port_ = ntohs(addr.sin_port);
    HttpServer* self = s.get();
    s->acceptor_ = std::jthread([self](std::stop_token st) { self->accept_loop(st); });
    return s;
}

HttpServer::~HttpServer() {
    {
        std::lock_guard<std::mutex> lk(clients_mu_);
        stopping_ = true;
    }
    acceptor_.request_stop();
    if (acceptor_.joinable()) acceptor_.join();
    if (listen_fd_ >= 0) ::close(listen_fd_);
    std::vector<Client> clients;
    {
        std::lock_guard<std::mutex> lk(clients_mu_);
        for (auto& st : open_) st->close();  // waiting clients return
        clients.swap(clients_);
    }
    clients.clear();  // joins them
}

void HttpServer::accept_loop(std::stop_token stop) {
    while (!stop.stop_requested()) {
        pollfd pfd{listen_fd_, POLLIN, 0};
        if (::poll(&pfd, 1, 100) <= 0) continue;
        const int fd = ::accept(listen_fd_, nullptr, nullptr);
        if (fd < 0) continue;
        // a silent or stalled peer cannot hold its thread forever
        timeval tv{10, 0};
        ::setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
        ::setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &tv, sizeof(tv));
        std::lock_guard<std::mutex> lk(clients_mu_);
        // finished client threads are joined here, so the list stays short
        std::erase_if(clients_, [](const Client& c) { return c.done->load(); });
        auto done = std::make_shared<std::atomic<bool>>(false);
        clients_.push_back(Client{done, std::jthread([this, fd, done] {
                                      handle_client(fd);
                                      ::close(fd);
                                      done->store(true);
                                  })});
    }
}

std::string HttpServer::metrics_json() {
    Metrics a;
    std::string gpus;
    double ttft_w = 0, iter_w = 0;
    for (int32_t g = 0; g < router_.num_gpus(); ++g) {
        const Metrics m = router_.metrics(g);
        a.uptime_secs = std::max(a.uptime_secs, m.uptime_secs);
        a.total_requests_received += m.total_requests_received;
        a.total_requests_completed += m.total_requests_completed;
        a.total_tokens_generated += m.total_tokens_generated;
        a.active_batch_size += m.active_batch_size;
        a.waiting_queue_depth += m.waiting_queue_depth;
        a.kv_cache_used_blocks += m.kv_cache_used_blocks;
        a.kv_cache_total_blocks += m.kv_cache_total_blocks;
        a.total_preemptions += m.total_preemptions;
        a.total_iterations += m.total_iterations;
        ttft_w += m.avg_ttft_ms * double(m.total_requests_completed);
        iter_w += m.avg_iteration_latency_ms * double(m.total_iterations);
        gpus += (g ? ",\n    " : "\n    ") + gpu_json(g, m);
    }
    a.uptime_secs = std::max(a.uptime_secs, 1e-6);
    a.throughput_tokens_per_sec = double(a.total_tokens_generated) / a.uptime_secs;
    a.kv_cache_utilization_pct =
        a.kv_cache_total_blocks ? 100.0 * double(a.kv_cache_used_blocks) /
                                      double(a.kv_cache_total_blocks)
                                : 0.0;
    a.avg_ttft_ms = a.total_requests_completed ? ttft_w / double(a.total_requests_completed) : 0;
    a.avg_iteration_latency_ms = a.total_iterations ? iter_w / double(a.total_iterations) : 0;
    std::string j = a.to_json();  // the reference's layout, then the per-GPU list
    j.pop_back();                 // the closing brace
    while (!j.empty() && is_space(j.back())) j.pop_back();
    return j + ",\n  \"gpus\": [" + gpus + "\n  ]\n}";
}

void HttpServer::handle_client(int fd) {
    std::string req;
    std::size_t body_at = 0;
    if (!read_request(fd, req, body_at)) return;
    const std::string_view r(req);
    if (r.starts_with("GET /health")) {
        send_all(fd, "HTTP/1.1 200 OK\r\nContent-Type: text/plain\r\nContent-Length: 2\r\n"
                     "Connection: close\r\n\r\nOK");
        return;
    }
    if (r.starts_with("GET /v1/metrics")) {
        const std::string json = metrics_json();
        send_all(fd, std::format("HTTP/1.1 200 OK\r\nContent-Type: application/json\r\n"
                                 "Content-Length: {}\r\nConnection: close\r\n\r\n{}",
                                 json.size(), json));
        return;
    }
    if (r.starts_with("POST /v1/generate")) {
        const std::string_view body = body_at <= r.size() ? r.substr(body_at) : "";
        const std::string prompt = json_string(body, "prompt", "cpp26 continuous batching");
        const std::size_t max_tokens = std::max<std::size_t>(json_usize(body, "max_tokens", 32), 1);
        if (!send_all(fd, "HTTP/1.1 200 OK\r\nContent-Type: text/event-stream\r\n"
                          "Cache-Control: no-cache\r\nConnection: keep-alive\r\n\r\n")) {
            return;
        }
        auto stream = std::make_shared<TokenStream>();
        {
            std::lock_guard<std::mutex> lk(clients_mu_);
            if (stopping_) return;  // no new requests while the server stops
            open_.push_back(stream);
        }
        const SeqId id = next_seq_.fetch_add(1);
        auto placed = router_.add_request(id, tokenize_prompt(prompt, cfg_.vocab_size),
                                          max_tokens, stream);
        if (placed) {
            while (auto ev = stream->pop_wait()) {
                std::string frame =
                    ev->ttft_us
                        ? std::format("data: {{\"seq_id\":{},\"token_id\":{},\"text\":\"{}\","
                                      "\"finished\":{},\"ttft_us\":{}}}\n\n",
                                      ev->seq_id, ev->token, token_text(ev->token),
                                      ev->finished ? "true" : "false", *ev->ttft_us)
                        : std::format("data: {{\"seq_id\":{},\"token_id\":{},\"text\":\"{}\","
                                      "\"finished\":{}}}\n\n",
                                      ev->seq_id, ev->token, token_text(ev->token),
                                      ev->finished ? "true" : "false");
                if (!send_all(fd, frame)) {
                    stream->close();  // the client went away; the request runs to its end
                    break;
                }
            }
            served_.fetch_add(1);
        }
        std::lock_guard<std::mutex> lk(clients_mu_);
        std::erase(open_, stream);
        return;
    }
    send_all(fd, "HTTP/1.1 404 Not Found\r\nContent-Length: 9\r\nConnection: close\r\n\r\nNot Found");
}

}  // namespace nvllm

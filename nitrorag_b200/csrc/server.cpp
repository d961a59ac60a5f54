// NitroRPC inference front end on the engine's C ABI (include/nitro_server.h).
//
// The reference's Server_Inference (src/Server_Inference.cpp) runs a TCP listener thread
// that reads one NitroRPC int vector per connection (src/NitroRPC.hpp:48-56) and queues a
// Request, and an engine loop that moves queued requests into Continuous_Scheduler, steps
// it and answers on each request's socket.  Here the same split: the listener thread reads
// and validates the prompt and queues (socket, prompt); nr_server_poll, on the thread that
// owns the engine, admits queued prompts with nr_add_request, runs one step (nr_step or a
// caller-supplied function with its contract) and streams every emitted token id, closing
// a connection once its request has finished.
#include <arpa/inet.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <sys/time.h>
#include <unistd.h>

#include <atomic>
#include <chrono>
#include <condition_variable>
#include <cstring>
#include <deque>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

#include "../../include/nitro_engine.h"
#include "../../include/nitro_server.h"

namespace {

// send_all / recv_all of src/NitroRPC.hpp:19-37; MSG_NOSIGNAL so that a client that went
// away makes send fail instead of raising SIGPIPE in the server process.
bool send_all(int fd, const void* buf, size_t len) {
    const char* p = static_cast<const char*>(buf);
    while (len > 0) {
        const ssize_t n = send(fd, p, len, MSG_NOSIGNAL);
        if (n <= 0) return false;
        p += n;
        len -= (size_t)n;
    }
    return true;
}

bool recv_all(int fd, void* buf, size_t len) {
    char* p = static_cast<char*>(buf);
    while (len > 0) {
        const ssize_t n = recv(fd, p, len, 0);
        if (n <= 0) return false;
        p += n;
        len -= (size_t)n;
    }
    return true;
}

struct Pending {
    int fd;
    std::vector<int32_t> prompt;
};

struct Client {
    int fd;  // -1 once the client is gone (its request still runs to completion)
};

constexpr int kEmitCap = 8192;  // > max decode rows (1024) + prompt chunks a step can complete

}  // namespace

struct nr_server {
    nr_engine* engine = nullptr;
    nr_step_fn step = nullptr;
    void* step_ctx = nullptr;
    int listen_fd = -1;
    int port = 0;
    int32_t vocab = 0, seq_len = 0;
    std::thread listener;
    std::atomic<bool> stopping{false};
    std::atomic<bool> run_stop{false};
    std::mutex mu;
    std::condition_variable cv;
    std::deque<Pending> queue;  // guarded by mu
    std::map<int32_t, Client> clients;
    int32_t next_id = 0;
    std::vector<int32_t> ids, toks;
    std::atomic<int64_t> accepted{0}, refused{0}, sent{0}, finished{0};

    void refuse(int fd) {
        close(fd);
        refused++;
    }

    // Listener thread (Server_Inference.cpp:16-37): accept, read one int vector, validate,
    // queue.  Polls with a timeout so nr_server_destroy can stop it.
    void listen_loop() {
        while (!stopping.load()) {
            pollfd p{listen_fd, POLLIN, 0};
            const int r = ::poll(&p, 1, 100);
            if (r <= 0 || !(p.revents & POLLIN)) continue;
            const int fd = accept(listen_fd, nullptr, nullptr);
            if (fd < 0) continue;
            timeval tv{5, 0};  // a client that sends nothing does not hold the listener
            setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
            int one = 1;
            setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));  // one small packet per token
            int32_t n = 0;
            if (!recv_all(fd, &n, sizeof(n)) || n <= 0 || n > seq_len) {
                refuse(fd);
                continue;
            }
            Pending item{fd, std::vector<int32_t>((size_t)n)};
            if (!recv_all(fd, item.prompt.data(), (size_t)n * sizeof(int32_t))) {
                refuse(fd);
                continue;
            }
            bool ok = true;
            for (int32_t t : item.prompt) ok = ok && t >= 0 && t < vocab;
            if (!ok) {
                refuse(fd);
                continue;
            }
            {
                std::lock_guard<std::mutex> lock(mu);
                queue.push_back(std::move(item));
            }
            accepted++;
            cv.notify_one();
        }
    }

    // Queued prompts -> scheduler (Server_Inference.cpp:94-99).
    int admit() {
        std::deque<Pending> batch;
        {
            std::lock_guard<std::mutex> lock(mu);
            batch.swap(queue);
        }
        for (Pending& p : batch) {
            const int32_t id = next_id++;
            const int rc = nr_add_request(engine, id, p.prompt.data(), (int32_t)p.prompt.size());
            if (rc != NR_OK) {
                refuse(p.fd);
                continue;
            }
            clients[id] = Client{p.fd};
        }
        return (int)batch.size();
    }

    int poll_once(int32_t wait_ms) {
        admit();
        int active = nr_has_active(engine);
        if (active < 0) return active;
        if (!active) {
            std::unique_lock<std::mutex> lock(mu);
            cv.wait_for(lock, std::chrono::milliseconds(std::max(wait_ms, 0)), [&] { return !queue.empty(); });
            lock.unlock();
            admit();
            active = nr_has_active(engine);
            if (active <= 0) return active < 0 ? active : 0;
        }
        nr_step_out out;
        std::memset(&out, 0, sizeof(out));
        out.emitted_cap = kEmitCap;
        out.emitted_req_ids = ids.data();
        out.emitted_tokens = toks.data();
        const int rc = step ? step(step_ctx, engine, &out) : nr_step(engine, &out);
        if (rc != NR_OK) return rc;
        const int n = std::min(out.n_emitted, kEmitCap);
        // stream each token as sampled (the reference's intent at :103-107)
        for (int i = 0; i < n; i++) {
            auto it = clients.find(ids[i]);
            if (it == clients.end() || it->second.fd < 0) continue;
            const int32_t tok = toks[i];
            if (send_all(it->second.fd, &tok, sizeof(tok))) {
                sent++;
            } else {
                close(it->second.fd);
                it->second.fd = -1;
            }
        }
        // close finished requests' connections (:108-110)
        for (int i = 0; i < n; i++) {
            auto it = clients.find(ids[i]);
            if (it == clients.end()) continue;
            int32_t flags[4] = {0, 0, 0, 0};
            if (nr_request_state(engine, ids[i], flags) == NR_OK && flags[2]) {
                if (it->second.fd >= 0) close(it->second.fd);
                clients.erase(it);
                finished++;
            }
        }
        return n;
    }
};

extern "C" {

int nr_server_create(nr_engine* e, const char* host, int32_t port, nr_step_fn step, void* step_ctx,
                     nr_server** out) {
    if (!e || !out || port < 0 || port > 65535) return NR_ERR_INVALID;
    int32_t shape[7];
    if (nr_model_shape(e, shape) != NR_OK) return NR_ERR_INVALID;
    sockaddr_in addr{};
    addr.sin_family = AF_INET;
    addr.sin_port = htons((uint16_t)port);
    if (!host) addr.sin_addr.s_addr = htonl(INADDR_ANY);
    else if (inet_pton(AF_INET, host, &addr.sin_addr) != 1) return NR_ERR_INVALID;
    const int fd = socket(AF_INET, SOCK_STREAM, 0);
    if (fd < 0) return NR_ERR_IO;
    int opt = 1;
    setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &opt, sizeof(opt));
    if (bind(fd, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) != 0 || listen(fd, 128) != 0) {
        close(fd);
        return NR_ERR_IO;
    }
    socklen_t len = sizeof(addr);
    getsockname(fd, reinterpret_cast<sockaddr*>(&addr), &len);
    nr_server* s = new nr_server();
    s->engine = e;
    s->step = step;
    s->step_ctx = step_ctx;
    s->listen_fd = fd;
    s->port = ntohs(addr.sin_port);
    s->vocab = shape[5];
    s->seq_len = shape[6];
    s->ids.resize(kEmitCap);
    s->toks.resize(kEmitCap);
    s->listener = std::thread([s] { s->listen_loop(); });
    *out = s;
    return NR_OK;
}

int nr_server_port(const nr_server* s) { return s ? s->port : NR_ERR_INVALID; }

int nr_server_poll(nr_server* s, int32_t wait_ms) {
    if (!s) return NR_ERR_INVALID;
    return s->poll_once(wait_ms);
}

int nr_server_run(nr_server* s) {
    if (!s) return NR_ERR_INVALID;
    s->run_stop = false;
    while (!s->run_stop.load()) {
        const int rc = s->poll_once(1);  // the reference idles in 1 ms sleeps (:113)
        if (rc < 0) return rc;
    }
    return NR_OK;
}

int nr_server_stop(nr_server* s) {
    if (!s) return NR_ERR_INVALID;
    s->run_stop = true;
    s->cv.notify_all();
    return NR_OK;
}

int nr_server_counters(const nr_server* s, int64_t counters4[4]) {
    if (!s || !counters4) return NR_ERR_INVALID;
    counters4[0] = s->accepted.load();
    counters4[1] = s->refused.load();
    counters4[2] = s->sent.load();
    counters4[3] = s->finished.load();
    return NR_OK;
}

int nr_server_destroy(nr_server* s) {
    if (!s) return NR_ERR_INVALID;
    s->stopping = true;
    if (s->listener.joinable()) s->listener.join();
    close(s->listen_fd);
    for (Pending& p : s->queue) close(p.fd);
    for (auto& kv : s->clients)
        if (kv.second.fd >= 0) close(kv.second.fd);
    delete s;
    return NR_OK;
}

}  // extern "C"

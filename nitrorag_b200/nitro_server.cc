// nitro_server: the inference server process (the reference's Server_Inference main,
// src/Server_Inference.cpp:39-116) on the engine's C ABI.
//
//   nitro_server MODEL.bin [--port 8081] [--device 0] [--blocks 1000] [--max-new 20]
//                [--packed] [--host 0.0.0.0]
//
// Loads the Q8_0 model file, creates the engine (pool of --blocks pages, as the
// reference's TOTAL_BLOCKS = 1000), serves NitroRPC prompts on --port (the reference's
// 8081) and streams every generated token.  SIGINT / SIGTERM stop the loop.
#include <csignal>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "../include/nitro_engine.h"
#include "../include/nitro_server.h"

static nr_server* g_server = nullptr;

static void on_signal(int) {
    if (g_server) nr_server_stop(g_server);
}

int main(int argc, char** argv) {
    if (argc < 2) {
        std::fprintf(stderr, "usage: %s MODEL.bin [--port P] [--device D] [--blocks N] [--max-new N] [--packed] [--host H]\n",
                     argv[0]);
        return 2;
    }
    nr_config cfg;
    nr_config_default(&cfg);
    cfg.total_blocks = 1000;
    cfg.device = 0;
    int port = 8081;
    const char* host = nullptr;
    for (int i = 2; i < argc; i++) {
        const bool more = i + 1 < argc;
        if (!std::strcmp(argv[i], "--port") && more) port = std::atoi(argv[++i]);
        else if (!std::strcmp(argv[i], "--device") && more) cfg.device = std::atoi(argv[++i]);
        else if (!std::strcmp(argv[i], "--blocks") && more) cfg.total_blocks = std::atoi(argv[++i]);
        else if (!std::strcmp(argv[i], "--max-new") && more) cfg.max_new_tokens = std::atoi(argv[++i]);
        else if (!std::strcmp(argv[i], "--host") && more) host = argv[++i];
        else if (!std::strcmp(argv[i], "--packed")) cfg.sched_mode = NR_SCHED_PACKED;
        else {
            std::fprintf(stderr, "unknown argument %s\n", argv[i]);
            return 2;
        }
    }
    nr_engine* e = nullptr;
    int rc = nr_engine_create(&cfg, argv[1], &e);
    if (rc != NR_OK) {
        std::fprintf(stderr, "nr_engine_create failed (%d): %s\n", rc, e ? nr_last_error(e) : "");
        return 1;
    }
    rc = nr_server_create(e, host, port, nullptr, nullptr, &g_server);
    if (rc != NR_OK) {
        std::fprintf(stderr, "nr_server_create failed (%d)\n", rc);
        nr_engine_destroy(e);
        return 1;
    }
    std::signal(SIGINT, on_signal);
    std::signal(SIGTERM, on_signal);
    std::printf("[nitro_server] listening on port %d\n", nr_server_port(g_server));
    std::fflush(stdout);
    rc = nr_server_run(g_server);
    if (rc != NR_OK) std::fprintf(stderr, "engine step failed (%d): %s\n", rc, nr_last_error(e));
    nr_server_destroy(g_server);
    nr_engine_destroy(e);
    return rc == NR_OK ? 0 : 1;
}

/* nitro_server.h — NitroRPC inference front end on the engine's C ABI.
 *
 * Replaces the reference's Server_Inference (nvivek17/NitroRAG src/Server_Inference.cpp:
 * 13-37 listener thread, :93-115 engine loop) and its NitroRPC framing
 * (src/NitroRPC.hpp:39-56, send_ints / recv_ints).  Wire format, as the reference and its
 * client (scripts/agent.py:62-70) use it, all values little-endian int32:
 *
 *   client -> server   n, then n prompt token ids        (one request per connection)
 *   server -> client   one token id per generated token, as soon as it is sampled;
 *                      the server closes the connection after the request's last token
 *
 * The reference streams nothing: its loop sends a token only when
 * Request::just_generated_new_token is set (Server_Inference.cpp:103-107), which no code
 * ever sets (src/pagedMemory.hpp:292).  This server sends every emitted token.  A prompt
 * that is empty, longer than the engine's sequence length or holds an id outside the
 * vocabulary is refused by closing the connection (the reference would index
 * prompt_tokens[0] of an empty prompt, pagedMemory.hpp:311).  A client that goes away
 * keeps its request running to completion; its tokens are dropped.
 *
 * Threads: one listener thread per server (accept + read the request, then queue it);
 * the engine loop runs on the thread that calls nr_server_poll / nr_server_run, which
 * must be the only thread driving the engine.
 */
#ifndef NITRO_SERVER_H
#define NITRO_SERVER_H

#include <stdint.h>

#include "nitro_engine.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct nr_server nr_server;

/* One scheduler iteration with the nr_step contract (the default is nr_step itself; a
 * host-only engine can be driven by a function that plans, samples and commits). */
typedef int (*nr_step_fn)(void* ctx, nr_engine* e, nr_step_out* out);

/* Bind host:port (host NULL = all interfaces, "127.0.0.1" = loopback; port 0 = any free
 * port) and start the listener thread.  step = NULL uses nr_step.  The engine must
 * outlive the server. */
int nr_server_create(nr_engine* e, const char* host, int32_t port, nr_step_fn step, void* step_ctx,
                     nr_server** out);
/* The bound TCP port. */
int nr_server_port(const nr_server* s);
/* One iteration of the engine loop (Server_Inference.cpp:93-115): move queued requests
 * into the scheduler, run one step if any request is active (otherwise wait up to
 * wait_ms for a request), send every emitted token to its client and close the
 * connections of finished requests.  Returns the number of tokens emitted (>= 0) or a
 * negative NR_ERR_* status from the step. */
int nr_server_poll(nr_server* s, int32_t wait_ms);
/* Loop nr_server_poll until nr_server_stop is called (from any thread); returns 0, or
 * the first negative status a step returned. */
int nr_server_run(nr_server* s);
int nr_server_stop(nr_server* s);
/* counters4 = requests accepted, requests refused, tokens sent, requests finished */
int nr_server_counters(const nr_server* s, int64_t counters4[4]);
/* Stop the listener, close every connection and free the server (not the engine). */
int nr_server_destroy(nr_server* s);

#ifdef __cplusplus
}
#endif
#endif /* NITRO_SERVER_H */

/*
 * A plain-C host of libprism_moe.so: built as C99 against include/prism_moe.h and linked to the
 * library, the way a non-Python integration (a C or C++ serving runtime, a cgo / JNI shim)
 * binds it. It makes only calls that need no GPU (version, size queries, argument checks) and
 * prints one line per check; the exit status is the number of failed checks.
 * Built and run by tests/test_abi.py.
 */
#include <stdio.h>
#include <string.h>

#include "prism_moe.h"

static int failures = 0;

static void check(int ok, const char* what) {
  printf("%s %s\n", ok ? "ok" : "FAIL", what);
  if (!ok) ++failures;
}

int main(void) {
  const int64_t T = 8192, H = 2048, I = 768;
  const int32_t E = 128, k = 8, W = 8;
  size_t land, ws;
  int st;

  check(prism_moe_version() >= 100, "version");
  check(prism_moe_dispatch_workspace_size(T, k, E, W) > 0, "dispatch workspace size");
  check(prism_moe_block_workspace_size(T, H, I, E, k, PRISM_MOE_BF16) > (size_t)(T * k * H * 2),
        "block workspace holds the permuted rows");
  check(prism_moe_block_workspace_size(-1, H, I, E, k, PRISM_MOE_BF16) == 0,
        "block workspace size rejects a negative token count");

  /* the landing zone receives up to W*T*k rows of H bf16 twice (two parities) */
  land = prism_moe_ep_landing_bytes(W, T, k, H, E, PRISM_MOE_BF16);
  check(land > (size_t)(2 * W * T * k * H * 2), "landing zone holds both receive parities");
  check(prism_moe_ep_landing_bytes(65, T, k, H, E, PRISM_MOE_BF16) == 0,
        "landing zone size rejects more than 64 ranks");
  ws = prism_moe_ep_workspace_size(T, H, I, E, k, W, PRISM_MOE_BF16);
  check(ws > 0, "EP workspace size");
  check(prism_moe_ep_workspace_size(T, H, I, 9, k, 2, PRISM_MOE_BF16) == 0,
        "EP workspace size rejects E % W != 0");
  check(prism_moe_ep_ipc_handle_bytes() > 0, "IPC handle size");

  st = prism_moe_route_topk(NULL, 7, 4, 8, 2, 1, NULL, NULL, NULL, NULL);
  check(st == PRISM_MOE_ERR_ARG && strstr(prism_moe_last_error(), "dtype") != NULL,
        "route_topk rejects an unknown dtype before touching the device");
  check(prism_moe_set_expert_engine(7) == PRISM_MOE_ERR_ARG, "engine outside the list");
  check(prism_moe_set_expert_engine(PRISM_MOE_ENGINE_AUTO) == PRISM_MOE_OK, "engine auto");
  check(prism_moe_set_wait_limits(-1, 0) == PRISM_MOE_ERR_ARG, "negative wait limit");
  check(prism_moe_set_wait_limits(0, 0) == PRISM_MOE_OK, "default wait limits");
  check(prism_moe_read_device_error(NULL, NULL) == PRISM_MOE_ERR_ARG,
        "read_device_error rejects a null word");
  return failures;
}

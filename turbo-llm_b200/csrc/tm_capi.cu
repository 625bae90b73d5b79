// C-ABI plumbing: error reporting, workspace layout, workspace init/status.
#include <stdarg.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <unordered_map>
#include <utility>

#include "tm_common.cuh"

namespace tmoe {

static thread_local char g_err[512] = "";

void set_error(const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

int fail(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int cuda_check(cudaError_t e, const char *what) {
  if (e == cudaSuccess) return TM_OK;
  return fail(TM_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorString(e), cudaGetErrorName(e));
}

static int64_t align_up(int64_t v, int64_t a) { return (v + a - 1) / a * a; }

bool pdl_enabled() {
  static const bool on = [] {
    const char *v = getenv("TM_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

int ensure_smem(const void *kernel, size_t dynamic_smem) {
  static std::mutex mu;
  static std::unordered_map<const void *, std::pair<size_t, size_t>> seen;  // static bytes, opted-in max
  std::lock_guard<std::mutex> g(mu);
  auto it = seen.find(kernel);
  if (it == seen.end()) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kernel);
    if (e != cudaSuccess) return cuda_check(e, "cudaFuncGetAttributes");
    it = seen.emplace(kernel, std::make_pair((size_t)fa.sharedSizeBytes, (size_t)0)).first;
  }
  if (it->second.first + dynamic_smem <= 48 * 1024 || dynamic_smem <= it->second.second) return TM_OK;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dynamic_smem);
  if (e != cudaSuccess) return cuda_check(e, "cudaFuncSetAttribute(max dynamic smem)");
  it->second.second = dynamic_smem;
  return TM_OK;
}

WsLayout ws_layout(int64_t tokens, int n_experts, int top_k, int hidden, int inter,
                   int shared_inter) {
  WsLayout L;
  memset(&L, 0, sizeof(L));
  const int64_t T = tokens, E = n_experts, P = tokens * top_k;
  const int64_t Is = shared_inter;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    int64_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  L.status = take(4);
  L.trace = take(kTraceBytes);  // right after the status word: offset independent of the shapes
  L.meta = take(8 * 4);
  L.router_cnt = take((kMaxTokenTiles + 1) * 4);
  L.k2_cnt = take((E + 1) * kMaxRG * 4);
  L.k3_cnt = take(kMaxRGo * 4);
  L.header_end = off;
  L.logits = take(T * E * 4);
  L.counts = take(E * 4);
  L.offsets = take((E + 1) * 4);
  L.act_list = take(E * 4);
  L.act_rec = take(E * 16);
  L.slot_token = take(P * 4);
  L.slot_pair = take(P * 4);
  L.pair_slot = take(P * 4);
  L.unit_hist = take((T + 15) / 16 * E * 4);
  L.sh_w = take(T * 4);
  L.h = take(P * inter * 4);
  L.sh_h = take(T * Is * 4);
  L.ypart = take((P + T) * hidden * 4);
  L.total = off;
  L.tokens = T;
  L.n_experts = n_experts;
  L.top_k = top_k;
  L.hidden = hidden;
  L.inter = inter;
  L.shared_inter = shared_inter;
  return L;
}

int ws_check(void *ws, int64_t ws_bytes, int64_t tokens, int n_experts, int top_k, int hidden,
             int inter, int shared_inter, WsLayout *L) {
  TM_REQUIRE(ws != nullptr, "workspace is NULL");
  TM_REQUIRE(aligned(ws, 256), "workspace must be 256-byte aligned");
  TM_REQUIRE(tokens >= 1, "tokens must be >= 1 (got %lld)", (long long)tokens);
  TM_REQUIRE(n_experts >= 1 && n_experts <= 1024, "n_experts %d outside [1, 1024]", n_experts);
  TM_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= n_experts, "top_k %d outside [1, min(32, E)]", top_k);
  TM_REQUIRE(hidden >= 128 && hidden <= kRows * kMaxRGo, "hidden %d outside [128, %d]", hidden,
             kRows * kMaxRGo);
  TM_REQUIRE(inter >= 0 && inter <= kRows * kMaxRG && shared_inter >= 0 && shared_inter <= kRows * kMaxRG,
             "inter (%d) and shared_inter (%d) must be <= %d", inter, shared_inter, kRows * kMaxRG);
  *L = ws_layout(tokens, n_experts, top_k, hidden, inter, shared_inter);
  if (ws_bytes < L->total)
    return fail(TM_ERR_WORKSPACE, "workspace has %lld bytes, call needs %lld", (long long)ws_bytes,
                (long long)L->total);
  return TM_OK;
}

}  // namespace tmoe

using namespace tmoe;

extern "C" int tm_abi_version(void) { return TM_ABI_VERSION; }

extern "C" const char *tm_last_error(void) { return g_err; }

extern "C" int64_t tm_workspace_bytes(int64_t max_tokens, int n_experts, int top_k, int hidden,
                                      int inter, int shared_inter) {
  if (max_tokens < 1 || n_experts < 1 || top_k < 1 || hidden < 1 || inter < 1 || shared_inter < 0)
    return -1;
  return ws_layout(max_tokens, n_experts, top_k, hidden, inter, shared_inter).total;
}

extern "C" int tm_plan_offsets(int64_t tokens, int n_experts, int top_k, int64_t *out8) {
  TM_REQUIRE(out8 != nullptr && tokens >= 1 && n_experts >= 1 && top_k >= 1, "bad arguments");
  const WsLayout L = ws_layout(tokens, n_experts, top_k, 128, 0, 0);
  const int64_t v[8] = {L.meta, L.counts, L.offsets, L.act_list, L.slot_token, L.slot_pair, L.pair_slot,
                        L.status};
  for (int i = 0; i < 8; ++i) out8[i] = v[i];
  return TM_OK;
}

#ifdef TM_TRACE
// Trace builds only: byte offset of the trace region in the workspace.
extern "C" int64_t tm_trace_offset(void) { return ws_layout(1, 1, 1, 128, 0, 0).trace; }
#endif

extern "C" int tm_workspace_init(void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(ws != nullptr && ws_bytes > 0, "workspace is NULL or empty");
  TM_REQUIRE(aligned(ws, 256), "workspace must be 256-byte aligned");
  return cuda_check(cudaMemsetAsync(ws, 0, static_cast<size_t>(ws_bytes), as_stream(stream)),
                    "tm_workspace_init memset");
}

extern "C" int tm_workspace_status(void *ws, int64_t ws_bytes, uint32_t *host_status, void *stream) {
  TM_REQUIRE(ws != nullptr && ws_bytes >= 4 && host_status != nullptr, "bad arguments");
  cudaStream_t s = as_stream(stream);
  int rc = cuda_check(cudaMemcpyAsync(host_status, ws, 4, cudaMemcpyDeviceToHost, s), "status copy");
  if (rc) return rc;
  rc = cuda_check(cudaStreamSynchronize(s), "status sync");
  if (rc) return rc;
  return cuda_check(cudaMemsetAsync(ws, 0, 4, s), "status clear");
}

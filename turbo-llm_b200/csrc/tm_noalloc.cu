// One whole MoE decode layer (router + gate/up + down/combine) whose scratch
// lives in a library-owned static device array instead of a caller workspace.
//
// Who needs this: callers that cannot allocate device memory for a workspace.
// A plain C or FFI host (cgo, JNI, ctypes without torch) often has no device
// allocator of its own, and a serving process whose memory pool has already
// claimed the free HBM for weights and KV pages cannot get a fresh buffer
// either; cudaMalloc/cudaFree would also synchronise the device and stall the
// other streams.  Such a caller passes only its inputs and outputs.
//
// The scratch is `tm_noalloc_scratch`, kNoAllocScratchBytes (8 MiB) per GPU,
// held by every GPU that loads the library until the process exits.  The
// kernels get its device address from cudaGetSymbolAddress, taken on the first
// call made with a device current and cached together with that device's
// current CUDA context: a call under another context (after cudaDeviceReset,
// or from a context the caller created itself) looks the address up again
// instead of reusing a stale one.  Every call shares
// the one array, which keeps the last call's contents: each call clears the
// header (status word and counters) before its kernels run.  Two calls that
// overlap on the GPU (different streams, or different host threads, on the
// same device) race on the array and give wrong results; order them on one
// stream.
#include <cuda.h>   // CUcontext (type only; cuCtxGetCurrent is reached through cudart)

#include <mutex>

#include "tm_common.cuh"

namespace {

constexpr int64_t kNoAllocScratchBytes = TM_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

// Host code sees this name only as a stand-in for the symbol; the device
// address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char tm_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
void *g_scratch_addr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

using CtxGetCurrentFn = CUresult (*)(CUcontext *);

// cuCtxGetCurrent through the runtime's driver entry point (the library links
// only the static CUDA runtime).  A thread on which no runtime call has yet
// made the device's context current reads NULL here; the caller then looks the
// address up again, and cudaGetSymbolAddress makes the context current.
int current_context(CUcontext *ctx) {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    int rc = tmoe::cuda_check(cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q),
                              "cudaGetDriverEntryPoint(cuCtxGetCurrent)");
    if (rc) return rc;
    if (!p || q != cudaDriverEntryPointSuccess)
      return tmoe::fail(TM_ERR_CUDA, "cuCtxGetCurrent is not available from the driver");
    fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  CUcontext c = nullptr;
  if (fn(&c) != CUDA_SUCCESS) return tmoe::fail(TM_ERR_CUDA, "cuCtxGetCurrent failed");
  *ctx = c;
  return TM_OK;
}

// Device address of the scratch on the current device (set-up on first use,
// and again whenever the device's current context has changed).
int scratch_on_current_device(void **out) {
  int dev = -1;
  int rc = tmoe::cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices)
    return tmoe::fail(TM_ERR_UNSUPPORTED, "device ordinal %d outside [0, %d)", dev, kMaxDevices);
  std::lock_guard<std::mutex> g(g_setup_mu);
  CUcontext ctx = nullptr;
  if (g_scratch_addr[dev]) {
    rc = current_context(&ctx);
    if (rc) return rc;
    if (ctx == g_scratch_ctx[dev]) {
      *out = g_scratch_addr[dev];
      return TM_OK;
    }
  }
  void *p = nullptr;
  rc = tmoe::cuda_check(cudaGetSymbolAddress(&p, tm_noalloc_scratch), "cudaGetSymbolAddress(tm_noalloc_scratch)");
  if (rc) return rc;
  if (!p || !tmoe::aligned(p, 256))
    return tmoe::fail(TM_ERR_CUDA, "static scratch address %p is not 256-byte aligned", p);
  rc = current_context(&ctx);   // the runtime has made the device's context current by now
  if (rc) return rc;
  g_scratch_addr[dev] = p;
  g_scratch_ctx[dev] = ctx;
  *out = p;
  return TM_OK;
}

}  // namespace

using namespace tmoe;

extern "C" int tm_moe_decode_layer_noalloc(
    const void *x, int64_t tokens, int hidden, int inter, int n_experts, int top_k, int act_dtype,
    const void *router_w, const uint8_t *w13, const float *s13, const uint8_t *w2, const float *s2,
    const uint8_t *sh_w13, const float *sh_s13, const uint8_t *sh_w2, const float *sh_s2,
    int shared_inter, const void *sh_gate_w, const void *residual, int64_t *topk_idx, void *topk_w,
    void *out, uint32_t *status, void *stream) {
  TM_REQUIRE(x && router_w && w13 && s13 && w2 && s2 && topk_idx && topk_w && out, "null pointer");
  TM_REQUIRE(tokens >= 1 && n_experts >= 1 && top_k >= 1 && hidden >= 128 && inter >= 1 && shared_inter >= 0,
             "bad shape (tokens %lld, E %d, top_k %d, hidden %d, inter %d, shared_inter %d)",
             (long long)tokens, n_experts, top_k, hidden, inter, shared_inter);
  TM_REQUIRE((sh_w13 == nullptr) == (sh_w2 == nullptr), "sh_w13 and sh_w2 must both be set or both be NULL");
  const WsLayout L = ws_layout(tokens, n_experts, top_k, hidden, inter, sh_w13 ? shared_inter : 0);
  if (L.total > kNoAllocScratchBytes)
    return fail(TM_ERR_WORKSPACE,
                "tm_moe_decode_layer_noalloc: this call needs %lld bytes of scratch but the static scratch "
                "holds %lld; use fewer tokens or the workspace entry points",
                (long long)L.total, (long long)kNoAllocScratchBytes);
  void *ws = nullptr;
  int rc = scratch_on_current_device(&ws);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  rc = cuda_check(cudaMemsetAsync(ws, 0, static_cast<size_t>(L.header_end), s), "scratch header clear");
  if (rc) return rc;
  const int is = sh_w13 ? shared_inter : 0;
  rc = tm_router_topk(x, tokens, hidden, act_dtype, router_w, n_experts, top_k, topk_idx, topk_w, nullptr, ws,
                      kNoAllocScratchBytes, stream);
  if (rc) return rc;
  // K2 with the down projections pulled into L2 for K3 (the variant the
  // workspace path uses; its results are identical to tm_moe_decode_gateup's)
  rc = tm_moe_decode_gateup_prefetch(x, tokens, hidden, inter, n_experts, top_k, act_dtype, w13, s13, sh_w13,
                                     sh_s13, is, sh_gate_w, w2, sh_w13 ? sh_w2 : nullptr, ws, kNoAllocScratchBytes,
                                     stream);
  if (rc) return rc;
  rc = tm_moe_decode_down_combine(tokens, hidden, inter, n_experts, top_k, act_dtype, topk_w, w2, s2, sh_w2,
                                  sh_s2, is, residual, out, ws, kNoAllocScratchBytes, stream);
  if (rc) return rc;
  if (status)
    return cuda_check(cudaMemcpyAsync(status, ws_ptr<char>(ws, L.status), 4, cudaMemcpyDeviceToDevice, s),
                      "status copy");
  return TM_OK;
}

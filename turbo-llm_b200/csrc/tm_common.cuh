// Shared device/host helpers for libturbomoe (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/turbomoe.h"

namespace tmoe {

// ---------------------------------------------------------------- errors ----
void set_error(const char *fmt, ...);
int fail(int code, const char *fmt, ...);
int cuda_check(cudaError_t e, const char *what);

#define TM_REQUIRE(cond, ...)                                  \
  do {                                                         \
    if (!(cond)) return ::tmoe::fail(TM_ERR_INVALID, __VA_ARGS__); \
  } while (0)

#define TM_LAUNCH_CHECK(what)                                                \
  do {                                                                       \
    cudaError_t _e = cudaGetLastError();                                     \
    if (_e != cudaSuccess) return ::tmoe::cuda_check(_e, what);                \
  } while (0)

inline cudaStream_t as_stream(void *s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ------------------------------------------------------------- act dtype ----
template <typename T> struct Act;
template <> struct Act<float> {
  static __device__ __forceinline__ float load(const float *p) { return *p; }
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Act<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};
template <> struct Act<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};

// Dispatch helper: calls f.template operator()<T>() for the act dtype code.
template <typename F> int dispatch_act(int dtype, F &&f) {
  switch (dtype) {
    case TM_DTYPE_F32: return f.template run<float>();
    case TM_DTYPE_F16: return f.template run<__half>();
    case TM_DTYPE_BF16: return f.template run<__nv_bfloat16>();
    default: return fail(TM_ERR_INVALID, "unknown act dtype %d", dtype);
  }
}

// ------------------------------------------------------------ e4m3 decode ----
// Two e4m3 bytes (low byte -> low half) to f16x2 with the hardware converter;
// every e4m3 value is exactly representable in f16.
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

// Four e4m3 bytes of a 32-bit word to four floats (byte 0 first), all exact.
// `volatile` keeps the conversions in program order, so a kernel that streams
// many 16-byte chunks decodes each one just before its FMAs instead of
// hoisting every decode (and its registers) ahead of the math.
__device__ __forceinline__ void e4m3x4_to_f32(uint32_t v, float &a, float &b, float &c, float &d) {
  asm volatile("{\n\t"
      ".reg .b16 q0, q1, h0, h1, h2, h3;\n\t"
      ".reg .b32 p0, p1;\n\t"
      "mov.b32 {q0, q1}, %4;\n\t"
      "cvt.rn.f16x2.e4m3x2 p0, q0;\n\t"
      "cvt.rn.f16x2.e4m3x2 p1, q1;\n\t"
      "mov.b32 {h0, h1}, p0;\n\t"
      "mov.b32 {h2, h3}, p1;\n\t"
      "cvt.f32.f16 %0, h0;\n\t"
      "cvt.f32.f16 %1, h1;\n\t"
      "cvt.f32.f16 %2, h2;\n\t"
      "cvt.f32.f16 %3, h3;\n\t"
      "}"
      : "=f"(a), "=f"(b), "=f"(c), "=f"(d)
      : "r"(v));
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t v) {
  uint32_t h = e4m3x2_to_f16x2(static_cast<uint16_t>(v));
  return __half2float(__ushort_as_half(static_cast<unsigned short>(h & 0xFFFFu)));
}

// ----------------------------------------------------------- memory ops ----
// Streaming 16-byte load of read-only weights (no L1 allocation).
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// L2-coherent loads for data written by other CTAs of the same grid.
__device__ __forceinline__ float ld_cg(const float *p) { return __ldcg(p); }
__device__ __forceinline__ int ld_cg(const int *p) { return __ldcg(p); }

__device__ __forceinline__ float silu(float g) { return g / (1.0f + __expf(-g)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// -------------------------------------------------------- workspace plan ----
// Byte offsets of the workspace regions.  The header (status, meta and all
// counters) depends only on the model shape, never on the token count, so the
// counters stay where tm_workspace_init zeroed them whatever T a call uses;
// the regions after it are laid out for the call's token count.
constexpr int kMaxTokenTiles = 4096;
constexpr int kMaxRG = 64;    // inter, shared_inter <= 2048 (row groups of 32)
constexpr int kMaxRGo = 512;  // hidden <= 16384

// The header and the plan regions depend only on (T, E, top_k), so the router
// (which does not know the expert sizes) and the expert kernels agree on them.

struct WsLayout {
  // header
  int64_t status;      // uint32 status word
  int64_t meta;        // int32[8]: n_active, pairs, tokens
  int64_t router_cnt;  // int32[kMaxTokenTiles + 1]: token-tile counters + tile-done counter
  int64_t k2_cnt;      // int32 [(E + 1) * kMaxRG]
  int64_t k3_cnt;      // int32 [kMaxRGo]
  int64_t header_end;
  // per-call regions
  int64_t logits;      // fp32 [T][E] (act-rounded logits)
  int64_t counts;      // int32 [E]
  int64_t offsets;     // int32 [E + 1]
  int64_t act_list;    // int32 [E]
  int64_t slot_token;  // int32 [P]
  int64_t slot_pair;   // int32 [P]
  int64_t pair_slot;   // int32 [P]
  int64_t gu_part;     // fp32 [KQ][P][2][I]
  int64_t sh_gu_part;  // fp32 [KQ][T][2][Is]
  int64_t shg_part;    // fp32 [KQ][T] shared-gate logit partials
  int64_t sh_w;        // fp32 [T] sigmoid(shared gate)
  int64_t h;           // fp32 [P][I]
  int64_t sh_h;        // fp32 [T][Is]
  int64_t ypart;       // fp32 [P + T][H]
  int64_t total;
  int64_t tokens;
  int n_experts, top_k, hidden, inter, shared_inter;
};

WsLayout ws_layout(int64_t tokens, int n_experts, int top_k, int hidden, int inter,
                   int shared_inter);

// Validate `ws` for a call with `tokens` tokens; fills *L.  Returns TM_OK or an error.
int ws_check(void *ws, int64_t ws_bytes, int64_t tokens, int n_experts, int top_k, int hidden,
             int inter, int shared_inter, WsLayout *L);

template <typename T> __host__ __device__ __forceinline__ T *ws_ptr(void *ws, int64_t off) {
  return reinterpret_cast<T *>(static_cast<char *>(ws) + off);
}

constexpr int kMetaNActive = 0;
constexpr int kMetaPairs = 1;
constexpr int kMetaTokens = 2;

}  // namespace tmoe

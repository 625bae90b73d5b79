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

// Opt `kernel` into `dynamic_smem` bytes of dynamic shared memory when its
// static plus dynamic shared memory exceeds the default 48 KB (cached per
// kernel; a host-side attribute, legal during stream capture).
int ensure_smem(const void *kernel, size_t dynamic_smem);

// Programmatic dependent launch is on unless TM_PDL=0 is set in the
// environment (read once; a launch-mode switch for measurements).
bool pdl_enabled();

// Launch with programmatic stream serialisation (PDL): the kernel may start
// while the previous kernel of the stream finishes; it must call pdl_wait()
// before touching anything that kernel writes.
template <typename Kern, typename... Args>
int launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const char *what,
               Args... args) {
  int rc = ensure_smem(reinterpret_cast<const void *>(kernel), smem);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cuda_check(cudaLaunchKernelEx(&cfg, kernel, args...), what);
}

inline bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ------------------------------------------------------------- act dtype ----
template <typename T> struct Act;
// Act<T>::ld_cg reads through L2 (never a possibly stale L1 line): used for
// every activation an earlier kernel of the same step wrote.
template <> struct Act<float> {
  static __device__ __forceinline__ float ld_cg(const float *p) { return __ldcg(p); }
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
  static __device__ __forceinline__ float round(float v) { return v; }
};
template <> struct Act<__half> {
  static __device__ __forceinline__ __half ld_cg(const __half *p) {
    return __ushort_as_half(__ldcg(reinterpret_cast<const unsigned short *>(p)));
  }
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
};
template <> struct Act<__nv_bfloat16> {
  static __device__ __forceinline__ __nv_bfloat16 ld_cg(const __nv_bfloat16 *p) {
    return __ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short *>(p)));
  }
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
// Streaming 16-byte load of read-only weights (no L1 allocation).  `volatile`
// keeps the loads where the kernel issues them (all of a tile up front), so
// they are in flight together instead of being sunk next to their first use.
__device__ __forceinline__ uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// ------------------------------------------- TMA bulk copies + mbarriers ----
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte asynchronous global -> shared copy through L2 of `src_bytes` bytes
// (16, or 0 to zero-fill the destination); completion by commit/wait groups.
__device__ __forceinline__ void cp_async16_z(uint32_t dst, const void *src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Make the initialised barrier visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// One contiguous global -> shared copy by the TMA unit (no multicast);
// completion is signalled on `bar` as transaction bytes.  src, dst 16-byte
// aligned, bytes a multiple of 16.
__device__ __forceinline__ void tma_bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 policy for weight streams read once per step: their lines are the first
// to be evicted, so the code, router weights, activations and workspace stay
// in L2 while gigabytes of expert weights pass through it.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// tma_bulk_g2s with an L2 cache policy (l2_evict_first for weight streams).
__device__ __forceinline__ void tma_bulk_g2s_hint(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                  uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Order this thread's earlier generic-proxy shared-memory accesses (after a
// CTA barrier: everyone's) before a following TMA write into the same bytes.
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// ------------------------------------------ cluster-scope mbarrier use ----
// Shared::cluster address of `p` (this CTA's shared variable) in the CTA of
// cluster rank `rank`.
__device__ __forceinline__ uint32_t cluster_addr(const void *p, int rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
// Asynchronous 4-byte store into shared memory of a CTA of the cluster; when
// it lands it completes 4 transaction bytes on that CTA's mbarrier, so the
// writer needs no fence and may exit right after issuing it.
__device__ __forceinline__ void st_async_u32(uint32_t dst_cluster_addr, uint32_t v, uint32_t bar_cluster_addr) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.u32 [%0], %1, [%2];" ::"r"(dst_cluster_addr),
               "r"(v), "r"(bar_cluster_addr)
               : "memory");
}
__device__ __forceinline__ void mbar_init_fence_cluster() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// Bounded wait with acquire at cluster scope: stores that other CTAs made
// before their release-arrive are visible after it returns true.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t *bar, uint32_t parity, uint64_t max_ns) {
  uint64_t t0 = 0;
  for (bool first = true;; first = false) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    if (ok) return true;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (first) t0 = t;
    else if (t - t0 > max_ns) return false;
  }
}

// Wait for phase `parity` of `bar` for at most ~`max_ns` nanoseconds of
// wall time (globaltimer).  Returns false on timeout; the caller records an
// error and abandons the work instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t max_ns = 1000000000ull) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    if (t - t0 > max_ns) return false;
  }
}

// ------------------------------------------ programmatic dependent launch ----
// Kernels launched with cudaLaunchAttributeProgrammaticStreamSerialization may
// start while the previous kernel in the stream still runs.  pdl_wait() blocks
// until that kernel has completed and its writes are visible; everything
// before it must touch only data no earlier kernel of the step writes
// (weights).  pdl_trigger() lets the next kernel start launching.  Both are
// no-ops for a normal launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// --------------------------------------------- warp-level tensor-core MMA ----
// Decode GEMVs run on mma.sync m16n8k16 (f16 x f16 -> f32): the 16-row packed
// chunk (16 rows x 16 bytes) is exactly one 16x16 A tile.  ldmatrix hands lane
// l bytes [4t, 4t+4) of row l/4 (t = l%4); mapping those four columns to the
// fragment's logical k = {2t, 2t+1, 2t+8, 2t+9} is a fixed permutation of the
// chunk's 16 columns, applied identically to the activations (B), so the dot
// products are unchanged and no register shuffling is needed.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t &r0, uint32_t &r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// Four e4m3 bytes (one ldmatrix word) -> two f16x2 words: bytes 0,1 -> lo, 2,3 -> hi.
__device__ __forceinline__ void e4m3x4_to_f16x2x2(uint32_t v, uint32_t &lo, uint32_t &hi) {
  asm("{\n\t.reg .b16 p, q;\n\tmov.b32 {p, q}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, p;\n\tcvt.rn.f16x2.e4m3x2 %1, q;\n\t}"
      : "=r"(lo), "=r"(hi)
      : "r"(v));
}

// d += A(16x32 e4m3) * B(32x8 e4m3), fp32 accumulators (products of two
// e4m3 values are exact in fp32).
__device__ __forceinline__ void mma_16832_e4m3(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.f32.e4m3.e4m3.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Power-of-2 exponent s that maps maxabs into [128, 256): v * 2^s then fits
// e4m3 (max 448) with its top bits in the normal range; 0 for maxabs 0.
__device__ __forceinline__ int e4m3_shift(float maxabs) {
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 0;
  int e;
  frexpf(maxabs, &e);
  return max(-100, min(100, 8 - e));
}

// Two fp32 -> two e4m3 bytes (a -> low byte, b -> high byte), and back.
__device__ __forceinline__ uint32_t e4m3x2_from(float a, float b) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(b), "f"(a));
  return r;
}
__device__ __forceinline__ float2 e4m3x2_value(uint32_t v) {
  uint32_t h;
  asm("{\n\t.reg .b16 p;\n\tcvt.u16.u32 p, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, p;\n\t}" : "=r"(h) : "r"(v));
  return __half22float2(*reinterpret_cast<__half2 *>(&h));
}

// Four scaled activations v (already multiplied by 2^s, |v| < 256) as three
// e4m3 terms, v ~= hi + mid / 16 + lo / 256, each term rounded to nearest:
// 12 significant bits, so a bf16 or fp16 value is kept to within 2^-12 of
// itself.  Bytes in element order, one u32 per term.
__device__ __forceinline__ void e4m3_split3(const float (&v)[4], uint32_t &hi, uint32_t &mid, uint32_t &lo) {
  float r[4];
  hi = e4m3x2_from(v[0], v[1]) | (e4m3x2_from(v[2], v[3]) << 16);
  {
    const float2 p = e4m3x2_value(hi & 0xFFFFu), q = e4m3x2_value(hi >> 16);
    r[0] = (v[0] - p.x) * 16.f;
    r[1] = (v[1] - p.y) * 16.f;
    r[2] = (v[2] - q.x) * 16.f;
    r[3] = (v[3] - q.y) * 16.f;
  }
  mid = e4m3x2_from(r[0], r[1]) | (e4m3x2_from(r[2], r[3]) << 16);
  {
    const float2 p = e4m3x2_value(mid & 0xFFFFu), q = e4m3x2_value(mid >> 16);
    r[0] = (r[0] - p.x) * 16.f;
    r[1] = (r[1] - p.y) * 16.f;
    r[2] = (r[2] - q.x) * 16.f;
    r[3] = (r[3] - q.y) * 16.f;
  }
  lo = e4m3x2_from(r[0], r[1]) | (e4m3x2_from(r[2], r[3]) << 16);
}

// d += A(16x16 f16) * B(16x8 f16), fp32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Exponent s so that maxabs * 2^-s lies in [2^13, 2^14): activations scaled by
// 2^-s are f16-representable exactly (bf16 / f16 inputs) with ample headroom
// for the fp32 accumulators; results are scaled back by 2^s (exact).
__device__ __forceinline__ int f16_shift(float maxabs) {
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 0;
  int e;
  frexpf(maxabs, &e);
  return max(-100, min(100, e - 14));
}

// ------------------------------------------------------------- tracing ----
// Builds with -DTM_TRACE record (kernel, event, CTA, globaltimer) per CTA into
// a workspace region, to reconstruct kernel timelines inside CUDA graphs.
// Product builds compile every hook to nothing and reserve no space.
#ifdef TM_TRACE
constexpr int64_t kTraceCap = 1 << 20;
constexpr int64_t kTraceBytes = 16 + kTraceCap * 16;
constexpr int kTraceSlots = 8;  // events a CTA may record per launch (ids 0..7)
// The CTA's first event (kTrEnter) reserves 2 * kTraceSlots entries with one
// atomic; later events are plain stores into them (no round trip), so the
// marks do not delay the code they time.  Event ev fills entry 2*ev with
// (header, globaltimer) and entry 2*ev+1 with (header | 0x80 << 48, clock64).
// Slots a CTA never writes keep the zeros the host cleared them to.
__device__ __forceinline__ void trace_event(uint32_t *tr, int kid, int ev) {
  __shared__ uint64_t *slot;
  if (tr && threadIdx.x == 0) {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    const uint64_t c = clock64();
    if (ev == 0) {
      const unsigned i = atomicAdd(tr, (unsigned)(2 * kTraceSlots));
      slot = i + 2 * kTraceSlots <= kTraceCap ? reinterpret_cast<uint64_t *>(tr + 4) + 2 * i : nullptr;
    }
    if (slot != nullptr && ev < kTraceSlots) {
      const uint64_t h = ((uint64_t)kid << 56) | ((uint64_t)ev << 48) | (uint64_t)(blockIdx.x + blockIdx.y * gridDim.x);
      slot[4 * ev] = h;
      slot[4 * ev + 1] = t;
      slot[4 * ev + 2] = h | (0x80ull << 48);
      slot[4 * ev + 3] = c;
    }
  }
}
#define TM_TRACE_EVENT(tr, kid, ev) ::tmoe::trace_event(tr, kid, ev)
#else
constexpr int64_t kTraceBytes = 0;
#define TM_TRACE_EVENT(tr, kid, ev) ((void)0)
#endif
enum { kTrRouter = 1, kTrGateUp = 2, kTrDown = 3, kTrDownT1 = 4, kTrPlan = 5 };
enum { kTrEnter = 0, kTrWaited = 1, kTrData = 2, kTrExit = 3 };

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
// Row-group height of the packed expert layout (tm_pack_experts): weights are
// stored as [row group][16-byte column chunk][rows of the group][16 bytes].
constexpr int kRows = 16;

constexpr int kMaxTokenTiles = 4096;
constexpr int kMaxRG = 128;    // inter, shared_inter <= 2048 (row groups of kRows)
constexpr int kMaxRGo = 1024;  // hidden <= 16384 (row groups of kRows)

// The header and the plan regions depend only on (T, E, top_k), so the router
// (which does not know the expert sizes) and the expert kernels agree on them.

struct WsLayout {
  // header
  int64_t status;      // uint32 status word
  int64_t meta;        // int32[8]: n_active, pairs, tokens
  int64_t router_cnt;  // int32[kMaxTokenTiles + 1]: token-tile counters + tile-done counter
  int64_t k2_cnt;      // int32 [(E + 1) * kMaxRG]
  int64_t k3_cnt;      // int32 [kMaxRGo]
  int64_t trace;       // kTraceBytes (0 in product builds)
  int64_t header_end;
  // per-call regions
  int64_t logits;      // fp32 [T][E] (act-rounded logits)
  int64_t counts;      // int32 [E]
  int64_t offsets;     // int32 [E + 1]
  int64_t act_list;    // int32 [E]
  int64_t act_rec;     // int4 [E]: {expert, count, first slot, 0} per active expert
  int64_t slot_token;  // int32 [P]
  int64_t slot_pair;   // int32 [P]
  int64_t pair_slot;   // int32 [P]
  int64_t unit_hist;   // int32 [ceil(T/16)][E]: routed pairs per expert of each 16-token unit
  int64_t sh_w;       // fp32 [T] sigmoid(shared gate)
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

// The grouped GEMMs (gate/up + SwiGLU, down) of tm_moe_prefill_grouped
// without the combine: per-slot expert outputs (act dtype, slot order) are
// left in the workspace's ypart region.  The plan must already be in `ws`.
int prefill_expert_outputs(const void *x, int64_t tokens, int hidden, int inter, int n_experts, int top_k,
                           int act_dtype, const uint8_t *w13, const float *s13, const uint8_t *w2, const float *s2,
                           void *ws, const WsLayout &L, cudaStream_t stream);

// The FP8 grouped GEMMs (tm_moe_f8.cu) for bf16 activations: per-slot expert
// outputs (bf16, slot order) in the ypart region, like prefill_expert_outputs.
int f8_expert_outputs(const void *x, int64_t T, int H, int I, int E, int k, const uint8_t *w13, const float *s13,
                      const uint8_t *w2, const float *s2, const uint8_t *sh_w13, const float *sh_s13,
                      const uint8_t *sh_w2, const float *sh_s2, const void *sh_gate_w, void *ws, const WsLayout &L,
                      cudaStream_t s);

// out[t] = sum_r topk_w[t,r] * y[pair_slot[t*k+r]] (top-k order, fp32) (+ sh_w[t] * y[sh_slot0 + t])
// (+ residual[t]), rounded once to act (k4_combine).
int combine_expert_outputs(const void *y, const void *topk_w, const int *pair_slot, const void *residual, void *out,
                           int64_t T, int H, int k, int act_dtype, const float *sh_w, int sh_slot0, cudaStream_t s);

constexpr int kMetaNActive = 0;
constexpr int kMetaPairs = 1;
constexpr int kMetaTokens = 2;

}  // namespace tmoe

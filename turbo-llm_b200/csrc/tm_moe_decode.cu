// K2 (gate+up dequant-GEMV + SwiGLU) and K3 (down dequant-GEMV + routing-
// weighted combine) for the decode path (1..64 tokens per layer call).
//
// Reference: moe_seq (execution/moe.py:7-20), the multi-token loop of
// MoEExecutor.execute_layer (moe.py:157-180) and the shared expert
// (moe.py:73-85, 191-202).
//
// A decode layer is latency-bound long before it is bandwidth-bound (38 MB in
// ~6 us), so each kernel keeps its chain of dependent memory round trips
// short and has no serial tail:
//   K2: a CTA owns one expert's 16 gate + 16 up rows over the whole hidden
//       dimension (one contiguous 32*H-byte tile of the packed layout, ONE TMA
//       bulk copy), so it produces final h = silu(g) * u itself;
//   K3 (one token): a CTA owns 16 output rows for every routed expert at once
//       (k tiles of 16*I bytes in flight together), combines them in shared
//       memory in top-k order and writes the output;
//   K3 (more tokens): a CTA owns (expert, 16 output rows); the last CTA of
//       each row group combines the experts.
// Lanes own weight rows (16 rows x 16 bytes = 256 contiguous bytes per
// chunk; two chunks per warp instruction, conflict-free), the activations
// they multiply come from shared memory as broadcasts, and block scales are
// per 16-column chunk (128x128 blocks).  Kernels are chained with
// programmatic dependent launch.
#include "tm_common.cuh"

namespace tmoe {

constexpr int kK2Warps = 4;                // K2: warps split the hidden dimension in 4
constexpr int kK2Threads = kK2Warps * 32;
constexpr int kK3Warps = 4;                // K3 general: 4 warps x 2 half-warps = 8 K slices
constexpr int kK3Threads = kK3Warps * 32;
constexpr int kK3T1Warps = 8;              // K3 one token: one warp per routed expert
constexpr int kK3T1Threads = kK3T1Warps * 32;
constexpr int kK3F8Warps = 16;             // one-token FP8 K3: two warps per expert (K halves)
constexpr int kK3F8Threads = kK3F8Warps * 32;
constexpr int kK3T1MaxExperts = 16;        // routed + shared experts the one-token path holds
constexpr int kK3T1MaxKB = 32;             // 128-column scale blocks per expert row it holds (K <= 4096)
constexpr int kCombineInKernelMaxT = 64;

struct PlanView {
  const int *meta;
  const int4 *act_rec;  // {expert, count, first slot, 0} per active expert
  const int *slot_token, *pair_slot;
  uint32_t *status;
  uint32_t *trace;  // trace builds only
};

static PlanView plan_view(void *ws, const WsLayout &L) {
  return PlanView{ws_ptr<int>(ws, L.meta),       ws_ptr<int4>(ws, L.act_rec),
                  ws_ptr<int>(ws, L.slot_token), ws_ptr<int>(ws, L.pair_slot),
                  ws_ptr<uint32_t>(ws, L.status), kTraceBytes ? ws_ptr<uint32_t>(ws, L.trace) : nullptr};
}

__device__ __forceinline__ int4 ld_cg4(const int4 *p) { return __ldcg(p); }

// All threads wait for phase `parity` of `bar`; the outcome is CTA-uniform.
// On timeout the status word is flagged and the CTA waits once more (bounded)
// for its copies to land before it may exit.
__device__ __forceinline__ bool tile_ready(uint64_t *bar, uint32_t *status, uint32_t parity = 0) {
  const bool ok = mbar_wait_bounded(bar, parity);
  if (__syncthreads_or(!ok)) {
    if (threadIdx.x == 0) {
      atomicOr(status, TM_STATUS_TIMEOUT);
      mbar_wait_bounded(bar, parity);
    }
    __syncthreads();
    return false;
  }
  return true;
}

// acc += (16 e4m3 weights of `v`) . x[0..16) for one token, x in shared memory.
__device__ __forceinline__ float dot_chunk(const uint4 &v, const float *x) {
  const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    float w0, w1, w2, w3;
    e4m3x4_to_f32(wv[q], w0, w1, w2, w3);
    const float4 xv = *reinterpret_cast<const float4 *>(x + q * 4);
    s = fmaf(w0, xv.x, s); s = fmaf(w1, xv.y, s); s = fmaf(w2, xv.z, s); s = fmaf(w3, xv.w, s);
  }
  return s;
}

// ===================================================================== K2 ====
template <typename TA> struct GateUpArgs {
  const TA *x;
  const uint8_t *w13;
  const float *s13;
  const uint8_t *sh_w13;
  const float *sh_s13;
  const TA *sh_gate_w;
  PlanView pl;
  float *sh_w, *h, *sh_h;
  // optional (NULL: none): the packed down projections of the same experts.
  // Once its own tile has landed, CTA (expert, row group rg) pulls bytes
  // [rg*16*H, (rg+1)*16*H) of that expert's w2 into L2; the RG = I/16 CTAs of
  // an expert cover its whole H x I down projection, so the K3 call that
  // follows reads it from L2 while HBM would otherwise idle through K2's
  // arithmetic and the kernel boundary.
  const uint8_t *pf_w2, *pf_sh_w2;
  int T, H, I, Is, E, P, RG, RGs;
  int routed_ctas;  // max_active * RG
};

// L2 prefetch of one 16-row slice of an expert's packed down projection
// (16 * H bytes, 16-byte aligned since H % 512 == 0); fire and forget.
__device__ __forceinline__ void k2_prefetch_down(const uint8_t *w2, int64_t expert_bytes, int expert, int rg,
                                                 int H) {
  if (w2 == nullptr) return;
  const uint8_t *p = w2 + (int64_t)expert * expert_bytes + (int64_t)rg * 16 * H;
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"((uint32_t)(16 * H)) : "memory");
}

template <typename TA, int kNT>
__global__ void __launch_bounds__(kK2Threads) k2_gateup(GateUpArgs<TA> a) {
  extern __shared__ __align__(128) uint8_t k2_smem[];
  const int tile_bytes = 32 * a.H;                                   // [H/16 chunks][2][16 rows][16 B]
  uint8_t *wtile = k2_smem;
  float *xs = reinterpret_cast<float *>(k2_smem + tile_bytes);       // [kNT][H]
  float *ssc = xs + kNT * a.H;                                       // [2][H/128] block scales
  __shared__ float red[kK2Warps][kNT][32];
  __shared__ float gred[kK2Warps][kNT];
  __shared__ __align__(8) uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrEnter);
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();  // the routing plan and x come from earlier kernels
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrWaited);
  int b = blockIdx.x;
  bool shared_expert;
  int rg, n, slot0, I, eid = 0;
  const uint8_t *wbase;
  const float *sbase;
  if (b < a.routed_ctas) {
    shared_expert = false;
    const int aidx = b / a.RG;
    rg = b % a.RG;
    const int n_active = ld_cg(a.pl.meta + kMetaNActive);
    const int4 rec = ld_cg4(a.pl.act_rec + aidx);  // issued together with n_active
    if (aidx >= n_active) return;
    n = rec.y;
    slot0 = rec.z;
    I = a.I;
    eid = rec.x;
    wbase = a.w13 + (int64_t)rec.x * 2 * a.I * a.H;
    sbase = a.s13 + (int64_t)rec.x * 2 * (a.I / 128) * (a.H / 128);
  } else {
    shared_expert = true;
    rg = b - a.routed_ctas;
    n = a.T;
    slot0 = 0;
    I = a.Is;
    wbase = a.sh_w13;
    sbase = a.sh_s13;
  }
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar, tile_bytes);
    tma_bulk_g2s_hint(wtile, wbase + (int64_t)rg * tile_bytes, tile_bytes, &bar, l2_evict_first());
  }
  pdl_trigger();
  const int HB = a.H / 128, KC = a.H / 16;
  const int ib = (rg * kRows) / 128;
  for (int i = tid; i < 2 * HB; i += kK2Threads) ssc[i] = __ldg(sbase + ib * 2 * HB + i);
  const int mat = lane >> 4;               // lanes 0-15: gate rows, 16-31: up rows
  const int cpw = KC / kK2Warps;           // chunks per warp
  const int kc0 = w * cpw;
  const uint8_t *wl = wtile + kc0 * 512 + lane * 16;
  const float *sl = ssc + mat * HB;

  for (int tg = 0; tg < n; tg += kNT) {
    const int nt = min(kNT, n - tg);
    if (tg) __syncthreads();  // xs / red reuse across token groups
    {
      // x rows as 16-byte vectors: all of a thread's loads are independent
      constexpr int V = 16 / sizeof(TA);
      const int vpt = a.H / V;
      int tok[kNT];
#pragma unroll
      for (int j = 0; j < kNT; ++j)
        tok[j] = (j >= nt) ? 0 : (shared_expert || a.T == 1) ? (tg + j) : ld_cg(a.pl.slot_token + slot0 + tg + j);
#pragma unroll
      for (int j = 0; j < kNT; ++j) {
        if (j < nt) {
          const uint4 *src = reinterpret_cast<const uint4 *>(a.x + (int64_t)tok[j] * a.H);
          for (int v = tid; v < vpt; v += kK2Threads) {
            const uint4 q = __ldcg(src + v);
            const TA *qe = reinterpret_cast<const TA *>(&q);
#pragma unroll
            for (int u = 0; u < V; ++u) xs[j * a.H + v * V + u] = Act<TA>::to_f(qe[u]);
          }
        }
      }
    }
    if (tg == 0) {
      if (!tile_ready(&bar, a.pl.status)) return;
      TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrData);
      if (tid == 0) {  // this CTA's tile is in: HBM can carry K3's weights now
        if (shared_expert) k2_prefetch_down(a.pf_sh_w2, (int64_t)a.H * a.Is, 0, rg, a.H);
        else k2_prefetch_down(a.pf_w2, (int64_t)a.H * a.I, eid, rg, a.H);
      }
    } else {
      __syncthreads();
    }
    float acc[kNT];
#pragma unroll
    for (int j = 0; j < kNT; ++j) acc[j] = 0.f;
    for (int blk = 0; blk < cpw / 8; ++blk) {  // 8 chunks = one 128-column scale block
      float bacc[kNT];
#pragma unroll
      for (int j = 0; j < kNT; ++j) bacc[j] = 0.f;
#pragma unroll 4
      for (int i = 0; i < 8; ++i) {
        const int kc = blk * 8 + i;
        const uint4 v = *reinterpret_cast<const uint4 *>(wl + kc * 512);
#pragma unroll
        for (int j = 0; j < kNT; ++j)
          if (j < nt) bacc[j] += dot_chunk(v, xs + j * a.H + (kc0 + kc) * 16);
      }
      const float sc = sl[(kc0 + blk * 8) / 8];
#pragma unroll
      for (int j = 0; j < kNT; ++j) acc[j] = fmaf(bacc[j], sc, acc[j]);
    }
#pragma unroll
    for (int j = 0; j < kNT; ++j) red[w][j][lane] = acc[j];
    if (shared_expert && rg == 0) {
      // shared-gate logit (moe.py:81-83): this warp's quarter of the columns
      for (int j = 0; j < nt; ++j) {
        float s = 0.f;
        for (int c = kc0 * 16 + lane; c < (kc0 + cpw) * 16; c += 32)
          s = fmaf(xs[j * a.H + c], Act<TA>::to_f(__ldg(a.sh_gate_w + c)), s);
        s = warp_sum(s);
        if (lane == 0) gred[w][j] = s;
      }
    }
    __syncthreads();
    if (tid < nt * kRows) {
      const int j = tid / kRows, r = tid % kRows;
      float g = 0.f, u = 0.f;
#pragma unroll
      for (int ww = 0; ww < kK2Warps; ++ww) {
        g += red[ww][j][r];
        u += red[ww][j][kRows + r];
      }
      float *hout = shared_expert ? a.sh_h : a.h;
      hout[(int64_t)(slot0 + tg + j) * I + rg * kRows + r] = silu(g) * u;
    }
    if (shared_expert && rg == 0 && tid < nt) {
      float s = 0.f;
#pragma unroll
      for (int ww = 0; ww < kK2Warps; ++ww) s += gred[ww][tid];
      // F.linear output and torch.sigmoid both produce the act dtype
      const float logit = Act<TA>::round(s);
      a.sh_w[tg + tid] = Act<TA>::round(1.0f / (1.0f + __expf(-logit)));
    }
  }
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrExit);
}

// Tensor-core K2 for 16-bit activations.  Each warp owns a quarter of the
// hidden dimension and waits only for its own quarter of the 32*H-byte tile
// (four TMA copies), so math starts while the rest of the tile streams in.
// Per 16-column chunk a warp issues one ldmatrix.x4 (gate rows 0-15, up rows
// 0-15), eight e4m3->f16x2 conversions and two m16n8k16 MMAs (N = up to 8
// tokens); block scales are applied per 8 chunks (128 columns).
template <typename TA, int kNT>
__global__ void __launch_bounds__(kK2Threads) k2_gateup_mma(GateUpArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  extern __shared__ __align__(128) uint8_t k2_smem[];
  const int tile_bytes = 32 * a.H;
  const int quarter = tile_bytes / kK2Warps;
  const int xstride = a.H + 8;  // f16 per staged token row (+16 bytes: no bank conflicts)
  uint8_t *wtile = k2_smem;
  // x rows land here as TA and are converted in place to f16; after the MMAs
  // the same bytes hold the cross-warp partial sums (keeps 3 CTAs per SM)
  __half *xs = reinterpret_cast<__half *>(k2_smem + tile_bytes);                 // [kNT][xstride]
  const TA *xraw = reinterpret_cast<const TA *>(xs);
  float *ssc = reinterpret_cast<float *>(k2_smem + tile_bytes + max(kNT * xstride * 2, 4096));  // [2][H/128]
  float(*red)[2][kRows][8] = reinterpret_cast<float(*)[2][kRows][8]>(xs);        // [kK2Warps] (4 KB)
  __shared__ float xmax[kK2Warps][kNT], s_gl[kK2Warps][kNT];
  __shared__ int s_shift[kNT];
  __shared__ __align__(8) uint64_t bar[kK2Warps];
  __shared__ __align__(8) uint64_t xbar;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrEnter);
  if (tid == 0) {
    for (int q = 0; q < kK2Warps; ++q) mbar_init(&bar[q], 1);
    mbar_init(&xbar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();  // the routing plan and x come from earlier kernels
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrWaited);
  int b = blockIdx.x;
  bool shared_expert;
  int rg, n, slot0, I, eid = 0;
  const uint8_t *wbase;
  const float *sbase;
  if (b < a.routed_ctas) {
    shared_expert = false;
    const int aidx = b / a.RG;
    rg = b % a.RG;
    const int n_active = ld_cg(a.pl.meta + kMetaNActive);
    const int4 rec = ld_cg4(a.pl.act_rec + aidx);  // issued together with n_active
    if (aidx >= n_active) return;
    n = rec.y;
    slot0 = rec.z;
    I = a.I;
    eid = rec.x;
    wbase = a.w13 + (int64_t)rec.x * 2 * a.I * a.H;
    sbase = a.s13 + (int64_t)rec.x * 2 * (a.I / 128) * (a.H / 128);
  } else {
    shared_expert = true;
    rg = b - a.routed_ctas;
    n = a.T;
    slot0 = 0;
    I = a.Is;
    wbase = a.sh_w13;
    sbase = a.sh_s13;
  }
  if (tid == 0) {
    const uint8_t *src = wbase + (int64_t)rg * tile_bytes;
    const uint64_t pol = l2_evict_first();
    for (int q = 0; q < kK2Warps; ++q) {
      mbar_arrive_expect_tx(&bar[q], quarter);
      tma_bulk_g2s_hint(wtile + q * quarter, src + q * quarter, quarter, &bar[q], pol);
    }
  }
  pdl_trigger();
  const int HB = a.H / 128, KC = a.H / 16;
  const int ib = (rg * kRows) / 128;
  for (int i = tid; i < 2 * HB; i += kK2Threads) ssc[i] = __ldg(sbase + ib * 2 * HB + i);
  const int cpw = KC / kK2Warps;  // chunks per warp
  const int kc0 = w * cpw;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t wsm = smem_u32(wtile) + kc0 * 512 + lane * 16;
  const bool gate_logit = shared_expert && rg == 0;
  bool first = true;

  for (int tg = 0, grp = 0; tg < n; tg += kNT, ++grp) {
    const int nt = min(kNT, n - tg);
    if (tg) __syncthreads();  // everyone is done with the previous group's x
    if (tid == 0) {
      fence_proxy_async();
      const uint32_t rowb = (uint32_t)a.H * sizeof(TA);
      mbar_arrive_expect_tx(&xbar, nt * rowb);
      for (int j = 0; j < nt; ++j) {
        const int tok = (shared_expert || a.T == 1) ? tg + j : ld_cg(a.pl.slot_token + slot0 + tg + j);
        tma_bulk_g2s(xs + (size_t)j * xstride, a.x + (int64_t)tok * a.H, rowb, &xbar);
      }
    }
    if (!tile_ready(&xbar, a.pl.status, grp & 1)) {
      if (tid == 0)
        for (int q = 0; q < kK2Warps; ++q) mbar_wait_bounded(&bar[q], 0);
      return;
    }
    // per-token max |x| -> exact power-of-2 shift; optional shared-gate logit (fp32)
    for (int j = 0; j < nt; ++j) {
      float m = 0.f, gl = 0.f;
      const int c_lo = w * (a.H / kK2Warps), c_hi = c_lo + a.H / kK2Warps;
      for (int c = c_lo + lane; c < c_hi; c += 32) {
        const float v = Act<TA>::to_f(xraw[(size_t)j * xstride + c]);
        m = fmaxf(m, fabsf(v));
        if (gate_logit) gl = fmaf(v, Act<TA>::to_f(__ldg(a.sh_gate_w + c)), gl);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (gate_logit) gl = warp_sum(gl);
      if (lane == 0) {
        xmax[w][j] = m;
        s_gl[w][j] = gl;
      }
    }
    __syncthreads();
    if (tid < nt) {
      float m = 0.f, gl = 0.f;
#pragma unroll
      for (int ww = 0; ww < kK2Warps; ++ww) {
        m = fmaxf(m, xmax[ww][tid]);
        gl += s_gl[ww][tid];
      }
      s_shift[tid] = f16_shift(m);
      if (gate_logit) {
        // F.linear output and torch.sigmoid both produce the act dtype (moe.py:81-83)
        const float logit = Act<TA>::round(gl);
        a.sh_w[tg + tid] = Act<TA>::round(1.0f / (1.0f + __expf(-logit)));
      }
    }
    __syncthreads();
    for (int i = tid; i < nt * (a.H / 2); i += kK2Threads) {  // in place: each pair read then written by one thread
      const int j = i / (a.H / 2), c = (i % (a.H / 2)) * 2;
      const float sc = ldexpf(1.0f, -s_shift[j]);
      const __half2 hv = __floats2half2_rn(Act<TA>::to_f(xraw[(size_t)j * xstride + c]) * sc,
                                           Act<TA>::to_f(xraw[(size_t)j * xstride + c + 1]) * sc);
      *reinterpret_cast<__half2 *>(xs + (size_t)j * xstride + c) = hv;
    }
    __syncthreads();
    if (first) {  // this warp's quarter of the weight tile
      first = false;
      const bool ok = mbar_wait_bounded(&bar[w], 0);
      if (__syncthreads_or(!ok)) {
        if (tid == 0) {
          atomicOr(a.pl.status, TM_STATUS_TIMEOUT);
          for (int q = 0; q < kK2Warps; ++q) mbar_wait_bounded(&bar[q], 0);
        }
        return;
      }
      TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrData);
      if (tid == 0) {  // this CTA's tile is in: HBM can carry K3's weights now
        if (shared_expert) k2_prefetch_down(a.pf_sh_w2, (int64_t)a.H * a.Is, 0, rg, a.H);
        else k2_prefetch_down(a.pf_w2, (int64_t)a.H * a.I, eid, rg, a.H);
      }
    }
    const __half *xrow = xs + (size_t)min(g, nt - 1) * xstride + 4 * t;  // B column n = g
    float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
    for (int blk = 0; blk < cpw / 8; ++blk) {
      float dg[4] = {0.f, 0.f, 0.f, 0.f}, du[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int kc = blk * 8 + i;
        uint32_t r0, r1, r2, r3, a0, a1, a2, a3;
        ldsm_x4(wsm + kc * 512, r0, r1, r2, r3);
        const uint2 bx = *reinterpret_cast<const uint2 *>(xrow + (kc0 + kc) * 16);
        e4m3x4_to_f16x2x2(r0, a0, a2);
        e4m3x4_to_f16x2x2(r1, a1, a3);
        mma_16816(dg, a0, a1, a2, a3, bx.x, bx.y);
        e4m3x4_to_f16x2x2(r2, a0, a2);
        e4m3x4_to_f16x2x2(r3, a1, a3);
        mma_16816(du, a0, a1, a2, a3, bx.x, bx.y);
      }
      const int cb = (kc0 + blk * 8) / 8;
      const float sg = ssc[cb], su = ssc[HB + cb];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        accg[q] = fmaf(dg[q], sg, accg[q]);
        accu[q] = fmaf(du[q], su, accu[q]);
      }
    }
    // D fragment: (row g, tokens 2t, 2t+1), (row g+8, tokens 2t, 2t+1); the
    // partial sums reuse the x staging bytes once every warp is past its MMAs
    TM_TRACE_EVENT(a.pl.trace, kTrGateUp, 4);  // warp 0's MMAs done
    __syncthreads();
    red[w][0][g][2 * t] = accg[0];
    red[w][0][g][2 * t + 1] = accg[1];
    red[w][0][g + 8][2 * t] = accg[2];
    red[w][0][g + 8][2 * t + 1] = accg[3];
    red[w][1][g][2 * t] = accu[0];
    red[w][1][g][2 * t + 1] = accu[1];
    red[w][1][g + 8][2 * t] = accu[2];
    red[w][1][g + 8][2 * t + 1] = accu[3];
    __syncthreads();
    if (tid < nt * kRows) {
      const int j = tid / kRows, r = tid % kRows;
      float gs = 0.f, us = 0.f;
#pragma unroll
      for (int ww = 0; ww < kK2Warps; ++ww) {
        gs += red[ww][0][r][j];
        us += red[ww][1][r][j];
      }
      const float back = ldexpf(1.0f, s_shift[j]);
      float *hout = shared_expert ? a.sh_h : a.h;
      hout[(int64_t)(slot0 + tg + j) * I + rg * kRows + r] = silu(gs * back) * (us * back);
    }
  }
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrExit);
}

// One-token K2 on FP8 tensor cores: mma.sync m16n8k32 e4m3 x e4m3 reads the
// packed weight tile as it is (no e4m3 -> f16 conversion), and the token
// enters as three e4m3 terms x * 2^s ~= hi + mid/16 + lo/256 (12 significant
// bits: within 2^-12 of each bf16/fp16 value), one per MMA column, so one MMA
// of 32 weight columns serves all three.  Half the MMAs of k2_gateup_mma and
// none of its conversions; fp32 accumulation, block scale per 128 columns.
// Shared memory: tile, the three e4m3 rows of x (the raw row lands over mid and
// lo first), block scales.
template <typename TA, int kW, int kSt>
__global__ void __launch_bounds__(kW * 32) k2_gateup_f8(GateUpArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  extern __shared__ __align__(128) uint8_t k2_smem[];
  const int tile_bytes = 32 * a.H;
  const int part = tile_bytes / kW;  // the slice of the tile each warp waits for
  uint8_t *wtile = k2_smem;
  // the three e4m3 term rows of x are XS = H + 16 bytes apart: the MMA B
  // loads of lanes reading the hi, mid and lo rows (same column) hit
  // different banks
  const int XS = a.H + 16;
  uint8_t *xb = k2_smem + tile_bytes;                          // [3][XS] e4m3: hi, mid, lo
  const TA *xraw = reinterpret_cast<const TA *>(xb + XS);      // [H] act (before the split)
  float *ssc = reinterpret_cast<float *>(xb + 3 * XS);         // [2][H/128]
  __shared__ float red[kW][2][kRows];
  __shared__ float xmax[kW], s_gl[kW];
  __shared__ int s_shift;
  __shared__ __align__(8) uint64_t bar[kW];
  __shared__ __align__(8) uint64_t xbar;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrEnter);
  if (tid == 0) {
    for (int q = 0; q < kW; ++q) mbar_init(&bar[q], 1);
    mbar_init(&xbar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  pdl_wait();  // the routing plan and x come from earlier kernels
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrWaited);
  int b = blockIdx.x;
  bool shared_expert;
  int rg, slot0, I, eid = 0;
  const uint8_t *wbase;
  const float *sbase;
  if (b < a.routed_ctas) {
    shared_expert = false;
    const int aidx = b / a.RG;
    rg = b % a.RG;
    const int n_active = ld_cg(a.pl.meta + kMetaNActive);
    const int4 rec = ld_cg4(a.pl.act_rec + aidx);  // issued together with n_active
    if (aidx >= n_active) return;
    slot0 = rec.z;
    I = a.I;
    eid = rec.x;
    wbase = a.w13 + (int64_t)rec.x * 2 * a.I * a.H;
    sbase = a.s13 + (int64_t)rec.x * 2 * (a.I / 128) * (a.H / 128);
  } else {
    shared_expert = true;
    rg = b - a.routed_ctas;
    slot0 = 0;
    I = a.Is;
    wbase = a.sh_w13;
    sbase = a.sh_s13;
  }
  if (tid == 0) {
    const uint8_t *src = wbase + (int64_t)rg * tile_bytes;
    const uint64_t pol = l2_evict_first();
    for (int q = 0; q < kW; ++q) {
      mbar_arrive_expect_tx(&bar[q], part);
      tma_bulk_g2s_hint(wtile + q * part, src + q * part, part, &bar[q], pol);
    }
    const uint32_t rowb = (uint32_t)a.H * sizeof(TA);
    mbar_arrive_expect_tx(&xbar, rowb);
    tma_bulk_g2s(const_cast<TA *>(xraw), a.x, rowb, &xbar);  // the single token
  }
  pdl_trigger();
  const int HB = a.H / 128, KC = a.H / 16;
  const int ib = (rg * kRows) / 128;
  for (int i = tid; i < 2 * HB; i += (kW * 32)) ssc[i] = __ldg(sbase + ib * 2 * HB + i);
  const bool gate_logit = shared_expert && rg == 0;
  if (!tile_ready(&xbar, a.pl.status, 0)) {
    if (tid == 0)
      for (int q = 0; q < kW; ++q) mbar_wait_bounded(&bar[q], 0);
    return;
  }
  // max |x| -> power-of-2 scale; optional shared-gate logit (fp32), same order
  // as k2_gateup_mma
  {
    float m = 0.f, gl = 0.f;
    const int c_lo = w * (a.H / kW), c_hi = c_lo + a.H / kW;
    for (int c = c_lo + lane; c < c_hi; c += 32) {
      const float v = Act<TA>::to_f(xraw[c]);
      m = fmaxf(m, fabsf(v));
      if (gate_logit) gl = fmaf(v, Act<TA>::to_f(__ldg(a.sh_gate_w + c)), gl);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (gate_logit) gl = warp_sum(gl);
    if (lane == 0) {
      xmax[w] = m;
      s_gl[w] = gl;
    }
  }
  __syncthreads();
  if (tid == 0) {
    float m = 0.f, gl = 0.f;
#pragma unroll
    for (int ww = 0; ww < kW; ++ww) {
      m = fmaxf(m, xmax[ww]);
      gl += s_gl[ww];
    }
    s_shift = e4m3_shift(m);
    if (gate_logit) {
      // F.linear output and torch.sigmoid both produce the act dtype (moe.py:81-83)
      const float logit = Act<TA>::round(gl);
      a.sh_w[0] = Act<TA>::round(1.0f / (1.0f + __expf(-logit)));
    }
  }
  __syncthreads();
  {  // split: every thread first reads its elements (the raw row overlaps mid/lo)
    constexpr int kMaxSteps = 8;  // H <= 4096 (host checks)
    const int steps = a.H / (4 * (kW * 32));
    const float sc = ldexpf(1.0f, s_shift);
    float v[kMaxSteps][4];
#pragma unroll
    for (int k = 0; k < kMaxSteps; ++k)
      if (k < steps) {
        const int c = 4 * (tid + k * (kW * 32));
#pragma unroll
        for (int u = 0; u < 4; ++u) v[k][u] = Act<TA>::to_f(xraw[c + u]) * sc;
      }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kMaxSteps; ++k)
      if (k < steps) {
        const int c = 4 * (tid + k * (kW * 32));
        uint32_t h, md, l;
        e4m3_split3(v[k], h, md, l);
        *reinterpret_cast<uint32_t *>(xb + c) = h;
        *reinterpret_cast<uint32_t *>(xb + XS + c) = md;
        *reinterpret_cast<uint32_t *>(xb + 2 * XS + c) = l;
      }
  }
  __syncthreads();
  const int cpw = KC / kW;  // 16-column chunks per warp
  const int kc0 = w * cpw;
  const int g = lane >> 2, t = lane & 3;
  // B column n = g: 0 hi, 1 mid, 2 lo (columns 3-7 repeat lo and are not read)
  const uint8_t *xsel = xb + min(g, 2) * XS + kc0 * 16 + 4 * t;
  // kSt > 0: the warp's kSt B fragment pairs in registers, loaded while the
  // weights are still in flight (the MMA loop then reads only the tile)
  uint32_t bx[kSt > 0 ? kSt : 1][2];
#pragma unroll
  for (int st = 0; st < kSt; ++st) {
    bx[st][0] = *reinterpret_cast<const uint32_t *>(xsel + st * 32);
    bx[st][1] = *reinterpret_cast<const uint32_t *>(xsel + st * 32 + 16);
  }
  // this warp's part of the weight tile: each warp starts its MMAs as soon as
  // its own part has landed (the parts arrive over microseconds); the CTA
  // agrees on a timeout at the reduction barrier below
  const bool part_ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bar[w], 0));
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrData);  // warp 0's part landed
  if (tid == 0 && part_ok) {  // HBM can carry K3's weights now
    if (shared_expert) k2_prefetch_down(a.pf_sh_w2, (int64_t)a.H * a.Is, 0, rg, a.H);
    else k2_prefetch_down(a.pf_w2, (int64_t)a.H * a.I, eid, rg, a.H);
  }
  // A (ldmatrix.x4): lanes 0-15 rows 0-15 of chunk kc, lanes 16-31 of chunk kc+1
  const uint32_t wsm = smem_u32(wtile) + (kc0 + (lane >> 4)) * 512 + (lane & 15) * 16;
  float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
  // (kSt > 0: cpw / 8 == kSt / 4, a compile-time trip count keeps bx in registers)
  const int nblk = part_ok ? (kSt > 0 ? kSt / 4 : cpw / 8) : 0;
#pragma unroll(kSt > 0 ? kSt / 4 : 2)
  for (int blk = 0; blk < (kSt > 0 ? kSt / 4 : cpw / 8); ++blk) {
    if (blk >= nblk) break;
    float dg[2][4], du[2][4];  // four independent MMA chains (two per operand)
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int q = 0; q < 4; ++q) dg[c][q] = du[c][q] = 0.f;
#pragma unroll
    for (int st = 0; st < 4; ++st) {
      const int kc = blk * 8 + 2 * st;
      uint32_t g0, g1, g2, g3, u0, u1, u2, u3;
      ldsm_x4(wsm + kc * 512, g0, g1, g2, g3);
      ldsm_x4(wsm + kc * 512 + 256, u0, u1, u2, u3);
      uint32_t b0, b1;
      if constexpr (kSt > 0) {
        b0 = bx[blk * 4 + st][0];
        b1 = bx[blk * 4 + st][1];
      } else {
        b0 = *reinterpret_cast<const uint32_t *>(xsel + kc * 16);
        b1 = *reinterpret_cast<const uint32_t *>(xsel + kc * 16 + 16);
      }
      mma_16832_e4m3(dg[st & 1], g0, g1, g2, g3, b0, b1);
      mma_16832_e4m3(du[st & 1], u0, u1, u2, u3, b0, b1);
    }
    const int cb = (kc0 + blk * 8) / 8;
    const float sg = ssc[cb], su = ssc[HB + cb];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      accg[q] = fmaf(dg[0][q] + dg[1][q], sg, accg[q]);
      accu[q] = fmaf(du[0][q] + du[1][q], su, accu[q]);
    }
  }
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, 4);  // warp 0's MMAs done
  // D: lane (g, t=0) holds columns hi, mid of rows g, g+8; lane (g, t=1) lo
  const float lg0 = __shfl_down_sync(0xffffffffu, accg[0], 1), lg8 = __shfl_down_sync(0xffffffffu, accg[2], 1);
  const float lu0 = __shfl_down_sync(0xffffffffu, accu[0], 1), lu8 = __shfl_down_sync(0xffffffffu, accu[2], 1);
  if (t == 0) {
    red[w][0][g] = accg[0] + (accg[1] + lg0 * 0.0625f) * 0.0625f;
    red[w][0][g + 8] = accg[2] + (accg[3] + lg8 * 0.0625f) * 0.0625f;
    red[w][1][g] = accu[0] + (accu[1] + lu0 * 0.0625f) * 0.0625f;
    red[w][1][g + 8] = accu[2] + (accu[3] + lu8 * 0.0625f) * 0.0625f;
  }
  if (__syncthreads_or(!part_ok)) {  // a part never landed: flag, let the copies finish, no output
    if (tid == 0) {
      atomicOr(a.pl.status, TM_STATUS_TIMEOUT);
      for (int q = 0; q < kW; ++q) mbar_wait_bounded(&bar[q], 0);
    }
    return;
  }
  if (tid < kRows) {
    float gs = 0.f, us = 0.f;
#pragma unroll
    for (int ww = 0; ww < kW; ++ww) {
      gs += red[ww][0][tid];
      us += red[ww][1][tid];
    }
    const float back = ldexpf(1.0f, -s_shift);
    float *hout = shared_expert ? a.sh_h : a.h;
    hout[(int64_t)slot0 * I + rg * kRows + tid] = silu(gs * back) * (us * back);
  }
  TM_TRACE_EVENT(a.pl.trace, kTrGateUp, kTrExit);
}

// =================================================================== K3 ====
template <typename TA> struct DownArgs {
  const TA *topk_w;
  const uint8_t *w2;
  const float *s2;
  const uint8_t *sh_w2;
  const float *sh_s2;
  const TA *residual;
  TA *out;
  PlanView pl;
  const float *h, *sh_h, *sh_w;
  float *ypart;  // [P + T][H]
  int *k3_cnt;
  int T, H, I, Is, E, k, P, RGo;
  int routed_ctas;  // max_active * RGo
  int has_shared;
  int combine_in_kernel;
  int tile_bytes;   // kRows * max(I, Is): shared-memory offset of the h staging area
};

// out[t, n] for rows [n0, n0 + nrows) and tokens [t0, t1): k-order weighted sum,
// then the gated shared expert, then the residual.
template <typename TA>
__device__ __forceinline__ void combine_rows(const DownArgs<TA> &a, int t0, int t1, int n0, int nrows,
                                             int tid, int nthreads) {
  constexpr int kMaxK = 16;  // ranks whose loads are issued together
  for (int i = tid; i < (t1 - t0) * nrows; i += nthreads) {
    const int t = t0 + i / nrows, nn = n0 + i % nrows;
    int slot[kMaxK];
    float wk[kMaxK], yv[kMaxK];
#pragma unroll
    for (int kk = 0; kk < kMaxK; ++kk) {
      slot[kk] = -1;
      wk[kk] = 0.f;
      if (kk < a.k) {
        slot[kk] = ld_cg(a.pl.pair_slot + (int64_t)t * a.k + kk);
        wk[kk] = Act<TA>::to_f(Act<TA>::ld_cg(a.topk_w + (int64_t)t * a.k + kk));
      }
    }
#pragma unroll
    for (int kk = 0; kk < kMaxK; ++kk)
      yv[kk] = slot[kk] >= 0 ? ld_cg(a.ypart + (int64_t)slot[kk] * a.H + nn) : 0.f;
    float y = 0.f;
#pragma unroll
    for (int kk = 0; kk < kMaxK; ++kk) y = fmaf(wk[kk], yv[kk], y);
    for (int kk = kMaxK; kk < a.k; ++kk) {
      const int s = ld_cg(a.pl.pair_slot + (int64_t)t * a.k + kk);
      if (s >= 0)
        y = fmaf(Act<TA>::to_f(Act<TA>::ld_cg(a.topk_w + (int64_t)t * a.k + kk)),
                 ld_cg(a.ypart + (int64_t)s * a.H + nn), y);
    }
    if (a.has_shared) y = fmaf(ld_cg(a.sh_w + t), ld_cg(a.ypart + (int64_t)(a.P + t) * a.H + nn), y);
    if (a.residual) y += Act<TA>::to_f(Act<TA>::ld_cg(a.residual + (int64_t)t * a.H + nn));
    a.out[(int64_t)t * a.H + nn] = Act<TA>::from_f(y);
  }
}

// One expert's 16 down rows against up to kNT tokens' h, K split in 8 slices
// (4 warps x 2 half-warps).  Lane: row = lane & 15, slice = 2 * warp + lane / 16.
template <int kNT>
__device__ __forceinline__ void down_rows_slices(const uint8_t *wtile, const float *hs, const float *srow,
                                                 int K, int nt, int w, int lane, float (&acc)[kNT]) {
  const int KC2 = K / 16;
  const int cps = KC2 / 8;                        // chunks per slice (K % 128 == 0)
  const int slice = w * 2 + (lane >> 4);
  const int kc0 = slice * cps;
  const uint8_t *wl = wtile + kc0 * 256 + (lane & 15) * 16;
#pragma unroll
  for (int j = 0; j < kNT; ++j) acc[j] = 0.f;
#pragma unroll 2
  for (int i = 0; i < cps; ++i) {
    const uint4 v = *reinterpret_cast<const uint4 *>(wl + i * 256);
    const float sc = __ldg(srow + (kc0 + i) / 8);
#pragma unroll
    for (int j = 0; j < kNT; ++j)
      if (j < nt) acc[j] = fmaf(dot_chunk(v, hs + j * K + (kc0 + i) * 16), sc, acc[j]);
  }
}

template <typename TA, int kNT>
__global__ void __launch_bounds__(kK3Threads) k3_down(DownArgs<TA> a) {
  extern __shared__ __align__(128) uint8_t k3_smem[];
  uint8_t *wtile = k3_smem;                                         // [K/16 chunks][16 rows][16 B]
  float *hs = reinterpret_cast<float *>(k3_smem + a.tile_bytes);    // [kNT][K]
  __shared__ float red[8][kNT][kRows];
  __shared__ __align__(8) uint64_t bar;   // weight tile
  __shared__ __align__(8) uint64_t hbar;  // h rows of the current token group (one phase per group)
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init(&hbar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  // The routing plan was written by the router, which completed before any K2
  // CTA passed its own griddepcontrol.wait, i.e. before this grid could start:
  // it may be read (through L2) ahead of this kernel's wait on K2.
  int b = blockIdx.x;
  const int n_active = ld_cg(a.pl.meta + kMetaNActive);
  bool shared_expert, idle = false;
  int rgo, n = 0, slot0 = 0, K;
  const uint8_t *wbase = nullptr;
  const float *sbase = nullptr;
  const float *hsrc = nullptr;
  if (b < a.routed_ctas) {
    shared_expert = false;
    const int aidx = b / a.RGo;
    rgo = b % a.RGo;
    K = a.I;
    if (aidx >= max(n_active, 1)) return;
    if (n_active == 0) {
      idle = true;  // no routed pair: still counted so that the combine runs
    } else {
      const int4 rec = ld_cg4(a.pl.act_rec + aidx);
      n = rec.y;
      slot0 = rec.z;
      wbase = a.w2 + (int64_t)rec.x * a.H * a.I;
      sbase = a.s2 + (int64_t)rec.x * (a.H / 128) * (a.I / 128);
      hsrc = a.h;
    }
  } else {
    shared_expert = true;
    rgo = b - a.routed_ctas;
    n = a.T;
    K = a.Is;
    wbase = a.sh_w2;
    sbase = a.sh_s2;
    hsrc = a.sh_h;
  }
  const int tile = kRows * K;
  if (!idle && tid == 0) {
    mbar_arrive_expect_tx(&bar, tile);
    tma_bulk_g2s_hint(wtile, wbase + (int64_t)rgo * tile, tile, &bar, l2_evict_first());
  }
  pdl_trigger();
  pdl_wait();  // K2 (h) has completed
  if (!idle) {
    const float *srow = sbase + (int64_t)((rgo * kRows) / 128) * (K / 128);
    const int ypbase = shared_expert ? a.P : 0;
    for (int tg = 0, grp = 0; tg < n; tg += kNT, ++grp) {
      const int nt = min(kNT, n - tg);
      if (tg) __syncthreads();  // every thread is done with the previous group's h
      if (tid == 0) {
        // h rows of consecutive slots are contiguous: one bulk copy per group
        fence_proxy_async();
        const uint32_t bytes = (uint32_t)nt * K * sizeof(float);
        mbar_arrive_expect_tx(&hbar, bytes);
        tma_bulk_g2s(hs, hsrc + (int64_t)(slot0 + tg) * K, bytes, &hbar);
      }
      if (tg == 0 && !tile_ready(&bar, a.pl.status)) {
        if (tid == 0) mbar_wait_bounded(&hbar, 0);
        return;
      }
      if (!tile_ready(&hbar, a.pl.status, grp & 1)) return;
      float acc[kNT];
      down_rows_slices<kNT>(wtile, hs, srow, K, nt, w, lane, acc);
#pragma unroll
      for (int j = 0; j < kNT; ++j) red[w * 2 + (lane >> 4)][j][lane & 15] = acc[j];
      __syncthreads();
      if (tid < nt * kRows) {
        const int j = tid / kRows, r = tid % kRows;
        float s = 0.f;
#pragma unroll
        for (int sl = 0; sl < 8; ++sl) s += red[sl][j][r];
        a.ypart[(int64_t)(ypbase + slot0 + tg + j) * a.H + rgo * kRows + r] = s;
      }
    }
  }
  if (!a.combine_in_kernel) return;
  // the last CTA of this row group (all experts) combines the 16 rows
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int *cnt = a.k3_cnt + rgo;
    const int prev = atomicAdd(cnt, 1);
    s_last = (prev == max(n_active, 1) + a.has_shared - 1);
    if (s_last) *cnt = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  combine_rows<TA>(a, 0, a.T, rgo * kRows, kRows, tid, kK3Threads);
}

// One token: a CTA owns 16 output rows and every routed expert (+ the shared
// one) at once; no partial outputs leave the CTA.
template <typename TA>
__global__ void __launch_bounds__(kK3T1Threads) k3_down_t1(DownArgs<TA> a) {
  extern __shared__ __align__(128) uint8_t k3_smem[];
  __shared__ float ysm[kK3T1MaxExperts][kRows];
  __shared__ int4 s_rec[kK3T1MaxExperts];
  __shared__ int s_slot[32], s_map[32];   // pair -> slot, slot -> active expert
  __shared__ float s_w[32];
  __shared__ __align__(8) uint64_t bar;   // weight tiles
  __shared__ __align__(8) uint64_t hbar;  // h of every slot
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int rgo = blockIdx.x;
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrEnter);
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init(&hbar, 1);
    mbar_fence_init();
  }
  // plan (the router completed before this grid could start, see k3_down)
  const int n_active = ld_cg(a.pl.meta + kMetaNActive);
  const int n_exp = n_active + a.has_shared;  // <= kK3T1MaxExperts (host checks the bound)
  if (tid < n_active) s_rec[tid] = ld_cg4(a.pl.act_rec + tid);
  if (tid < a.k) {
    s_slot[tid] = ld_cg(a.pl.pair_slot + tid);
    s_w[tid] = Act<TA>::to_f(Act<TA>::ld_cg(a.topk_w + tid));
  }
  __syncthreads();
  const int tile_r = kRows * a.I, tile_s = kRows * a.Is;
  // [routed tiles][shared tile][h of the k slots][shared h]
  float *hs = reinterpret_cast<float *>(k3_smem + (size_t)n_active * tile_r + tile_s);
  if (tid < n_active)
    for (int c = 0; c < s_rec[tid].y; ++c) s_map[s_rec[tid].z + c] = tid;
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar, n_active * tile_r + (a.has_shared ? tile_s : 0));
    for (int e = 0; e < n_active; ++e)
      tma_bulk_g2s_hint(k3_smem + (size_t)e * tile_r,
                        a.w2 + (int64_t)s_rec[e].x * a.H * a.I + (int64_t)rgo * tile_r, tile_r, &bar,
                        l2_evict_first());
    if (a.has_shared)
      tma_bulk_g2s_hint(k3_smem + (size_t)n_active * tile_r, a.sh_w2 + (int64_t)rgo * tile_s, tile_s, &bar,
                        l2_evict_first());
  }
  pdl_trigger();
  pdl_wait();  // K2 (h) has completed
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrWaited);
  if (tid == 0) {
    const uint32_t hb = (uint32_t)a.k * a.I * sizeof(float), hsb = (uint32_t)a.Is * sizeof(float);
    mbar_arrive_expect_tx(&hbar, hb + (a.has_shared ? hsb : 0));
    tma_bulk_g2s(hs, a.h, hb, &hbar);  // slots 0..k-1 of the single token
    if (a.has_shared) tma_bulk_g2s(hs + (size_t)a.k * a.I, a.sh_h, hsb, &hbar);
  }
  const bool ok = mbar_wait_bounded(&bar, 0) & mbar_wait_bounded(&hbar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      atomicOr(a.pl.status, TM_STATUS_TIMEOUT);
      mbar_wait_bounded(&bar, 0);
      mbar_wait_bounded(&hbar, 0);
    }
    return;
  }
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrData);
  for (int e = w; e < n_exp; e += kK3T1Warps) {
    const bool sh = e == n_active;
    const int K = sh ? a.Is : a.I;
    const uint8_t *wt = k3_smem + (size_t)e * tile_r;  // the shared tile follows the routed ones
    const float *he = sh ? hs + (size_t)a.k * a.I : hs + (size_t)s_rec[e].z * a.I;
    const float *srow = (sh ? a.sh_s2 : a.s2 + (int64_t)s_rec[e].x * (a.H / 128) * (a.I / 128)) +
                        (int64_t)((rgo * kRows) / 128) * (K / 128);
    // lane: row = lane & 15, half of K = lane / 16
    const int cph = K / 32;  // chunks per half
    const int kc0 = (lane >> 4) * cph;
    const uint8_t *wl = wt + kc0 * 256 + (lane & 15) * 16;
    float acc = 0.f;
#pragma unroll 4
    for (int i = 0; i < cph; ++i) {
      const uint4 v = *reinterpret_cast<const uint4 *>(wl + i * 256);
      acc = fmaf(dot_chunk(v, he + (kc0 + i) * 16), __ldg(srow + (kc0 + i) / 8), acc);
    }
    acc += __shfl_xor_sync(0xffffffffu, acc, 16);
    if (lane < kRows) ysm[e][lane] = acc;
  }
  __syncthreads();
  if (tid < kRows) {
    float y = 0.f;
    for (int kk = 0; kk < a.k; ++kk)
      if (s_slot[kk] >= 0) y = fmaf(s_w[kk], ysm[s_map[s_slot[kk]]][tid], y);
    if (a.has_shared) y = fmaf(ld_cg(a.sh_w), ysm[n_active][tid], y);
    const int nn = rgo * kRows + tid;
    if (a.residual) y += Act<TA>::to_f(Act<TA>::ld_cg(a.residual + nn));
    a.out[nn] = Act<TA>::from_f(y);
  }
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrExit);
}

// Tensor-core one-token K3 for 16-bit activations: warp e multiplies expert
// e's 16 x I tile by that expert's h (converted to f16 with an exact
// power-of-2 shift), one ldmatrix.x2 + four conversions + one m16n8k16 MMA
// per 16-column chunk (only column 0 of N carries the token).
template <typename TA>
__global__ void __launch_bounds__(kK3T1Threads) k3_down_t1_mma(DownArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  extern __shared__ __align__(128) uint8_t k3_smem[];
  __shared__ float ysm[kK3T1MaxExperts][kRows];
  __shared__ float s_sc[kK3T1MaxExperts][kK3T1MaxKB];  // block scales of this CTA's 16 rows
  __shared__ float s_back[kK3T1MaxExperts];            // 2^shift that undoes h's f16 scaling
  __shared__ int4 s_rec[kK3T1MaxExperts];
  __shared__ int s_slot[32], s_map[32];   // pair -> slot, slot -> active expert
  __shared__ float s_w[32];
  __shared__ __align__(8) uint64_t bar;   // weight tiles
  __shared__ __align__(8) uint64_t hbar;  // h of every slot
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int rgo = blockIdx.x;
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrEnter);
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init(&hbar, 1);
    mbar_fence_init();
  }
  // plan (the router completed before this grid could start, see k3_down)
  const int n_active = ld_cg(a.pl.meta + kMetaNActive);
  const int n_exp = n_active + a.has_shared;  // <= kK3T1MaxExperts (host checks the bound)
  if (tid < n_active) s_rec[tid] = ld_cg4(a.pl.act_rec + tid);
  if (tid < a.k) {
    s_slot[tid] = ld_cg(a.pl.pair_slot + tid);
    s_w[tid] = Act<TA>::to_f(Act<TA>::ld_cg(a.topk_w + tid));
  }
  __syncthreads();
  const int tile_r = kRows * a.I, tile_s = kRows * a.Is;
  const int Kmax = max(a.I, a.Is), hstride = Kmax + 8;
  // [routed tiles][shared tile][h fp32: k slots x I, then Is][h f16: one row per expert]
  float *hs = reinterpret_cast<float *>(k3_smem + (size_t)n_active * tile_r + tile_s);
  __half *h16 = reinterpret_cast<__half *>(hs + (size_t)a.k * a.I + a.Is);
  if (tid < n_active)
    for (int c = 0; c < s_rec[tid].y; ++c) s_map[s_rec[tid].z + c] = tid;
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar, n_active * tile_r + (a.has_shared ? tile_s : 0));
    for (int e = 0; e < n_active; ++e)
      tma_bulk_g2s_hint(k3_smem + (size_t)e * tile_r,
                        a.w2 + (int64_t)s_rec[e].x * a.H * a.I + (int64_t)rgo * tile_r, tile_r, &bar,
                        l2_evict_first());
    if (a.has_shared)
      tma_bulk_g2s_hint(k3_smem + (size_t)n_active * tile_r, a.sh_w2 + (int64_t)rgo * tile_s, tile_s, &bar,
                        l2_evict_first());
  }
  // block scales into shared memory now (weights: independent of K2), not
  // one dependent global load per 128 columns inside the MMA loop
  {
    const int KB = a.I / 128, KBs = a.Is / 128, rb = (rgo * kRows) / 128;
    for (int i = tid; i < n_exp * kK3T1MaxKB; i += kK3T1Threads) {
      const int e = i / kK3T1MaxKB, b = i % kK3T1MaxKB;
      if (e == n_active) {
        if (b < KBs) s_sc[e][b] = __ldg(a.sh_s2 + (int64_t)rb * KBs + b);
      } else if (b < KB) {
        s_sc[e][b] = __ldg(a.s2 + ((int64_t)s_rec[e].x * (a.H / 128) + rb) * KB + b);
      }
    }
  }
  // the residual (this layer's input, complete before the router that
  // preceded K2 could pass its own wait) is loaded now, off the tail
  float res_pre = 0.f;
  if (tid < kRows && a.residual) res_pre = Act<TA>::to_f(Act<TA>::ld_cg(a.residual + rgo * kRows + tid));
  pdl_trigger();
  pdl_wait();  // K2 (h) has completed
  const float shw = (a.has_shared && tid < kRows) ? ld_cg(a.sh_w) : 0.f;  // gate score from K2
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrWaited);
  if (tid == 0) {
    const uint32_t hb = (uint32_t)a.k * a.I * sizeof(float), hsb = (uint32_t)a.Is * sizeof(float);
    mbar_arrive_expect_tx(&hbar, hb + (a.has_shared ? hsb : 0));
    tma_bulk_g2s(hs, a.h, hb, &hbar);  // slots 0..k-1 of the single token
    if (a.has_shared) tma_bulk_g2s(hs + (size_t)a.k * a.I, a.sh_h, hsb, &hbar);
  }
  const bool hok = mbar_wait_bounded(&hbar, 0);
  if (__syncthreads_or(!hok)) {
    if (tid == 0) {
      atomicOr(a.pl.status, TM_STATUS_TIMEOUT);
      mbar_wait_bounded(&bar, 0);
      mbar_wait_bounded(&hbar, 0);
    }
    return;
  }
  const int g = lane >> 2, t = lane & 3;
  for (int e = w; e < n_exp; e += kK3T1Warps) {
    const bool sh = e == n_active;
    const int K = sh ? a.Is : a.I;
    const float *hf = sh ? hs + (size_t)a.k * a.I : hs + (size_t)s_rec[e].z * a.I;
    __half *hh = h16 + (size_t)e * hstride;
    // this expert's h -> f16 with an exact power-of-2 shift (warp-local);
    // K % 128 == 0, so each lane's loads come in groups of 4 (issued together)
    float m4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int c = lane; c < K; c += 128) {
#pragma unroll
      for (int u = 0; u < 4; ++u) m4[u] = fmaxf(m4[u], fabsf(hf[c + 32 * u]));
    }
    float m = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int sh_exp = f16_shift(m);
    const float sc = ldexpf(1.0f, -sh_exp);
    if (lane == 0) s_back[e] = ldexpf(1.0f, sh_exp);
#pragma unroll 2
    for (int c = lane * 2; c < K; c += 128) {
      const float2 v0 = *reinterpret_cast<const float2 *>(hf + c);
      const float2 v1 = *reinterpret_cast<const float2 *>(hf + c + 64);
      *reinterpret_cast<__half2 *>(hh + c) = __floats2half2_rn(v0.x * sc, v0.y * sc);
      *reinterpret_cast<__half2 *>(hh + c + 64) = __floats2half2_rn(v1.x * sc, v1.y * sc);
    }
    __syncwarp();
  }
  const bool ok = mbar_wait_bounded(&bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      atomicOr(a.pl.status, TM_STATUS_TIMEOUT);
      mbar_wait_bounded(&bar, 0);
    }
    return;
  }
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrData);
  for (int e = w; e < n_exp; e += kK3T1Warps) {
    const bool sh = e == n_active;
    const int K = sh ? a.Is : a.I;
    const float back = s_back[e];  // written by this warp in the conversion pass
    const __half *hrow = h16 + (size_t)e * hstride + 4 * t;
    const uint32_t wsm = smem_u32(k3_smem + (size_t)e * tile_r) + (lane & 15) * 16;
    const float *srow = s_sc[e];
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int blk = 0; blk < K / 128; ++blk) {
      // four independent MMA chains of two 16-column chunks each
      float d[4][4];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int q = 0; q < 4; ++q) d[c][q] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int kc = blk * 8 + i;
        uint32_t r0, r1, a0, a1, a2, a3;
        ldsm_x2(wsm + kc * 256, r0, r1);
        const uint2 bx = *reinterpret_cast<const uint2 *>(hrow + kc * 16);
        e4m3x4_to_f16x2x2(r0, a0, a2);
        e4m3x4_to_f16x2x2(r1, a1, a3);
        mma_16816(d[i & 3], a0, a1, a2, a3, bx.x, bx.y);
      }
      const float s = srow[blk];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = fmaf((d[0][q] + d[1][q]) + (d[2][q] + d[3][q]), s, acc[q]);
    }
    // column 0 of D lives in lanes with t == 0: rows g (acc[0]) and g + 8 (acc[2])
    if (t == 0) {
      ysm[e][g] = acc[0] * back;
      ysm[e][g + 8] = acc[2] * back;
    }
  }
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, 4);  // warp 0's MMAs done
  __syncthreads();
  if (tid < kRows) {
    float y = 0.f;
    for (int kk = 0; kk < a.k; ++kk)
      if (s_slot[kk] >= 0) y = fmaf(s_w[kk], ysm[s_map[s_slot[kk]]][tid], y);
    if (a.has_shared) y = fmaf(shw, ysm[n_active][tid], y);
    const int nn = rgo * kRows + tid;
    if (a.residual) y += res_pre;
    a.out[nn] = Act<TA>::from_f(y);
  }
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrExit);
}

// One-token K3 on FP8 tensor cores: as k3_down_t1_mma, but each expert's h
// (fp32 from K2) enters as three e4m3 terms h * 2^s ~= hi + mid/16 + lo/256
// (12 significant bits; the per-expert power-of-2 s from max |h|), one per MMA
// column, and the packed e4m3 down tile is multiplied as it is by
// mma.sync m16n8k32: half the MMAs, no weight conversion.
template <typename TA>
__global__ void __launch_bounds__(kK3F8Threads) k3_down_t1_f8(DownArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  extern __shared__ __align__(128) uint8_t k3_smem[];
  __shared__ float ysm[kK3T1MaxExperts][2][kRows];   // per expert and K half
  __shared__ float s_sc[kK3T1MaxExperts][kK3T1MaxKB];  // block scales of this CTA's 16 rows
  __shared__ float s_back[kK3T1MaxExperts];            // 2^-shift that undoes h's scaling
  __shared__ int4 s_rec[kK3T1MaxExperts];
  __shared__ int s_slot[32], s_map[32];   // pair -> slot, slot -> active expert
  __shared__ float s_w[32];
  __shared__ __align__(8) uint64_t bar;   // weight tiles
  __shared__ __align__(8) uint64_t hbar;  // h of every slot
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int rgo = blockIdx.x;
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrEnter);
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init(&hbar, 1);
    mbar_fence_init();
  }
  // plan (the router completed before this grid could start, see k3_down)
  const int n_active = ld_cg(a.pl.meta + kMetaNActive);
  const int n_exp = n_active + a.has_shared;  // <= kK3T1MaxExperts (host checks the bound)
  if (tid < n_active) s_rec[tid] = ld_cg4(a.pl.act_rec + tid);
  if (tid < a.k) {
    s_slot[tid] = ld_cg(a.pl.pair_slot + tid);
    s_w[tid] = Act<TA>::to_f(Act<TA>::ld_cg(a.topk_w + tid));
  }
  __syncthreads();
  const int tile_r = kRows * a.I, tile_s = kRows * a.Is;
  const int Kmax = max(a.I, a.Is);
  // term rows of h, 16 bytes apart in bank order: the MMA B loads of lanes
  // reading the hi, mid and lo rows (same column) hit different banks
  const int KS = Kmax + 16;
  // [routed tiles][shared tile][h fp32: k slots x I, then Is][h e4m3: 3 x KS per expert]
  float *hs = reinterpret_cast<float *>(k3_smem + (size_t)n_active * tile_r + tile_s);
  uint8_t *h8 = reinterpret_cast<uint8_t *>(hs + (size_t)a.k * a.I + a.Is);
  if (tid < n_active)
    for (int c = 0; c < s_rec[tid].y; ++c) s_map[s_rec[tid].z + c] = tid;
  if (tid == 0) {
    mbar_arrive_expect_tx(&bar, n_active * tile_r + (a.has_shared ? tile_s : 0));
    for (int e = 0; e < n_active; ++e)
      tma_bulk_g2s_hint(k3_smem + (size_t)e * tile_r,
                        a.w2 + (int64_t)s_rec[e].x * a.H * a.I + (int64_t)rgo * tile_r, tile_r, &bar,
                        l2_evict_first());
    if (a.has_shared)
      tma_bulk_g2s_hint(k3_smem + (size_t)n_active * tile_r, a.sh_w2 + (int64_t)rgo * tile_s, tile_s, &bar,
                        l2_evict_first());
  }
  // block scales into shared memory now (weights: independent of K2), not
  // one dependent global load per 128 columns inside the MMA loop
  {
    const int KB = a.I / 128, KBs = a.Is / 128, rb = (rgo * kRows) / 128;
    for (int i = tid; i < n_exp * kK3T1MaxKB; i += kK3F8Threads) {
      const int e = i / kK3T1MaxKB, b = i % kK3T1MaxKB;
      if (e == n_active) {
        if (b < KBs) s_sc[e][b] = __ldg(a.sh_s2 + (int64_t)rb * KBs + b);
      } else if (b < KB) {
        s_sc[e][b] = __ldg(a.s2 + ((int64_t)s_rec[e].x * (a.H / 128) + rb) * KB + b);
      }
    }
  }
  // the residual (this layer's input, complete before the router that
  // preceded K2 could pass its own wait) is loaded now, off the tail
  float res_pre = 0.f;
  if (tid < kRows && a.residual) res_pre = Act<TA>::to_f(Act<TA>::ld_cg(a.residual + rgo * kRows + tid));
  pdl_trigger();
  pdl_wait();  // K2 (h) has completed
  const float shw = (a.has_shared && tid < kRows) ? ld_cg(a.sh_w) : 0.f;  // gate score from K2
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrWaited);
  // h (K2's output, in L2): for inner sizes up to 1024 each expert's warp
  // loads its row straight into registers (one L2 round trip, no CTA-wide
  // wait); larger rows come in by TMA into shared memory first
  const bool hreg = max(a.I, a.Is) <= 1024;
  if (tid == 0 && !hreg) {
    const uint32_t hb = (uint32_t)a.k * a.I * sizeof(float), hsb = (uint32_t)a.Is * sizeof(float);
    mbar_arrive_expect_tx(&hbar, hb + (a.has_shared ? hsb : 0));
    tma_bulk_g2s(hs, a.h, hb, &hbar);  // slots 0..k-1 of the single token
    if (a.has_shared) tma_bulk_g2s(hs + (size_t)a.k * a.I, a.sh_h, hsb, &hbar);
  }
  const bool hok = hreg || mbar_wait_bounded(&hbar, 0);
  if (__syncthreads_or(!hok)) {
    if (tid == 0) {
      atomicOr(a.pl.status, TM_STATUS_TIMEOUT);
      mbar_wait_bounded(&bar, 0);
      mbar_wait_bounded(&hbar, 0);
    }
    return;
  }
  const int g = lane >> 2, t = lane & 3;
  for (int e = w; e < n_exp; e += kK3F8Warps) {
    const bool sh = e == n_active;
    const int K = sh ? a.Is : a.I;
    const float *hf = sh ? hs + (size_t)a.k * a.I : hs + (size_t)s_rec[e].z * a.I;
    uint8_t *he = h8 + (size_t)e * 3 * KS;
    if (hreg) {  // lane owns elements 4 lane + 128 u (K % 128 == 0, K <= 1024)
      const float *hg = sh ? a.sh_h : a.h + (size_t)s_rec[e].z * a.I;
      float4 hv[8];
      float m = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (4 * lane + 128 * u < K) hv[u] = __ldcg(reinterpret_cast<const float4 *>(hg + 4 * lane + 128 * u));
#pragma unroll
      for (int u = 0; u < 8; ++u)
        if (4 * lane + 128 * u < K)
          m = fmaxf(m, fmaxf(fmaxf(fabsf(hv[u].x), fabsf(hv[u].y)), fmaxf(fabsf(hv[u].z), fabsf(hv[u].w))));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      const int sh_exp = e4m3_shift(m);
      const float sc = ldexpf(1.0f, sh_exp);
      if (lane == 0) s_back[e] = ldexpf(1.0f, -sh_exp);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int c = 4 * lane + 128 * u;
        if (c < K) {
          float v[4] = {hv[u].x * sc, hv[u].y * sc, hv[u].z * sc, hv[u].w * sc};
          uint32_t th, tm, tl;
          e4m3_split3(v, th, tm, tl);
          *reinterpret_cast<uint32_t *>(he + c) = th;
          *reinterpret_cast<uint32_t *>(he + KS + c) = tm;
          *reinterpret_cast<uint32_t *>(he + 2 * KS + c) = tl;
        }
      }
      __syncwarp();
      continue;
    }
    // this expert's h -> three e4m3 terms with a power-of-2 scale (warp-local);
    // K % 128 == 0, so each lane's loads come in groups of 4 (issued together)
    float m4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int c = lane; c < K; c += 128) {
#pragma unroll
      for (int u = 0; u < 4; ++u) m4[u] = fmaxf(m4[u], fabsf(hf[c + 32 * u]));
    }
    float m = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    const int sh_exp = e4m3_shift(m);
    const float sc = ldexpf(1.0f, sh_exp);
    if (lane == 0) s_back[e] = ldexpf(1.0f, -sh_exp);
#pragma unroll 2
    for (int c = 4 * lane; c < K; c += 128) {
      const float4 q = *reinterpret_cast<const float4 *>(hf + c);
      float v[4] = {q.x * sc, q.y * sc, q.z * sc, q.w * sc};
      uint32_t th, tm, tl;
      e4m3_split3(v, th, tm, tl);
      *reinterpret_cast<uint32_t *>(he + c) = th;
      *reinterpret_cast<uint32_t *>(he + KS + c) = tm;
      *reinterpret_cast<uint32_t *>(he + 2 * KS + c) = tl;
    }
    __syncwarp();
  }
  const bool ok = mbar_wait_bounded(&bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      atomicOr(a.pl.status, TM_STATUS_TIMEOUT);
      mbar_wait_bounded(&bar, 0);
    }
    return;
  }
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrData);
  // work items (expert, K half): warp w takes items w, w + 16, ...; item i is
  // expert i / 2, half i % 2 (128-column blocks [0, nb/2) and [nb/2, nb))
  for (int item = w; item < 2 * n_exp; item += kK3F8Warps) {
    const int e = item >> 1, half = item & 1;
    const bool sh = e == n_active;
    const int K = sh ? a.Is : a.I;
    const int nb = K / 128, nb0 = (nb + 1) / 2;
    const int blk_lo = half ? nb0 : 0, blk_hi = half ? nb : nb0;
    const float back = s_back[e];  // written in the conversion pass (a CTA barrier ago)
    // A (ldmatrix.x4): lanes 0-15 rows 0-15 of chunk kc, lanes 16-31 of chunk kc+1
    const uint32_t wsm = smem_u32(k3_smem + (size_t)e * tile_r) + (lane >> 4) * 256 + (lane & 15) * 16;
    // B column n = g: 0 hi, 1 mid, 2 lo (columns 3-7 repeat lo and are not read)
    const uint8_t *hsel = h8 + (size_t)e * 3 * KS + min(g, 2) * KS + 4 * t;
    const float *srow = s_sc[e];
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int blk = blk_lo; blk < blk_hi; ++blk) {
      float d[4][4];  // four independent MMA chains, one 32-column step each
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int q = 0; q < 4; ++q) d[c][q] = 0.f;
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        const int kc = blk * 8 + 2 * st;
        uint32_t a0, a1, a2, a3;
        ldsm_x4(wsm + kc * 256, a0, a1, a2, a3);
        const uint32_t b0 = *reinterpret_cast<const uint32_t *>(hsel + kc * 16);
        const uint32_t b1 = *reinterpret_cast<const uint32_t *>(hsel + kc * 16 + 16);
        mma_16832_e4m3(d[st], a0, a1, a2, a3, b0, b1);
      }
      const float s = srow[blk];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = fmaf((d[0][q] + d[1][q]) + (d[2][q] + d[3][q]), s, acc[q]);
    }
    // D: lane (g, t=0) holds columns hi, mid of rows g (acc[0], acc[1]) and
    // g + 8 (acc[2], acc[3]); lane (g, t=1) holds lo in acc[0], acc[2]
    const float lo0 = __shfl_down_sync(0xffffffffu, acc[0], 1), lo8 = __shfl_down_sync(0xffffffffu, acc[2], 1);
    if (t == 0) {
      ysm[e][half][g] = (acc[0] + (acc[1] + lo0 * 0.0625f) * 0.0625f) * back;
      ysm[e][half][g + 8] = (acc[2] + (acc[3] + lo8 * 0.0625f) * 0.0625f) * back;
    }
  }
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, 4);  // warp 0's MMAs done
  __syncthreads();
  if (tid < kRows) {
    float y = 0.f;
    for (int kk = 0; kk < a.k; ++kk)
      if (s_slot[kk] >= 0) {
        const int e = s_map[s_slot[kk]];
        y = fmaf(s_w[kk], ysm[e][0][tid] + ysm[e][1][tid], y);
      }
    if (a.has_shared) y = fmaf(shw, ysm[n_active][0][tid] + ysm[n_active][1][tid], y);
    const int nn = rgo * kRows + tid;
    if (a.residual) y += res_pre;
    a.out[nn] = Act<TA>::from_f(y);
  }
  TM_TRACE_EVENT(a.pl.trace, kTrDownT1, kTrExit);
}

template <typename TA>
__global__ void __launch_bounds__(256) k3_combine(DownArgs<TA> a) {
  // grid: (H / 16, ceil(T / 16)); 16 tokens x 16 rows per CTA
  pdl_wait();
  const int t0 = blockIdx.y * 16, t1 = min(a.T, t0 + 16);
  combine_rows<TA>(a, t0, t1, blockIdx.x * kRows, kRows, threadIdx.x, blockDim.x);
}

// ================================================================= launch ====
// Tokens per pass over a weight tile: an expert never has more tokens than the call.
static int tokens_per_pass(int64_t T, int cap) {
  const int t = T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : 8;
  return t < cap ? t : cap;
}

struct GateUpLaunch {
  const void *x; int64_t T; int H, I, E, k, Is;
  const uint8_t *w13; const float *s13; const uint8_t *sh_w13; const float *sh_s13; const void *sh_gate_w;
  void *ws; const WsLayout *L; cudaStream_t s;
  const uint8_t *pf_w2 = nullptr, *pf_sh_w2 = nullptr;  // down projections to pull into L2 (optional)
  template <typename TA, int kNT> int go(GateUpArgs<TA> &a, int grid) {
    if constexpr (sizeof(TA) == 2) {
      if (kNT == 1 && T == 1 && H <= 4096) {  // one token: FP8 MMAs on the split activation
        // 8 warps (H % 1024 == 0) split the reduction dimension finer: the
        // MMA chains of one warp are latency-bound, not the tensor pipe
        // (H = 1024 / 2048 / 3072 / 4096: the B fragments in registers)
        const size_t smem = (size_t)32 * H + (size_t)3 * (H + 16) + 2 * (H / 128) * sizeof(float);
        switch (H) {
          case 1024: return launch_pdl(k2_gateup_f8<TA, 8, 4>, dim3(grid), dim3(256), smem, s, "k2_gateup launch", a);
          case 2048: return launch_pdl(k2_gateup_f8<TA, 8, 8>, dim3(grid), dim3(256), smem, s, "k2_gateup launch", a);
          case 3072: return launch_pdl(k2_gateup_f8<TA, 8, 12>, dim3(grid), dim3(256), smem, s, "k2_gateup launch", a);
          case 4096: return launch_pdl(k2_gateup_f8<TA, 8, 16>, dim3(grid), dim3(256), smem, s, "k2_gateup launch", a);
          default: break;
        }
        return launch_pdl(k2_gateup_f8<TA, 4, 0>, dim3(grid), dim3(4 * 32), smem, s, "k2_gateup launch", a);
      }
      // tile + x rows (f16, padded; >= the 4 KB reduction area) + block scales
      const size_t smem = (size_t)32 * H + std::max<size_t>((size_t)kNT * (H + 8) * 2, 4096) +
                          2 * (H / 128) * sizeof(float);
      return launch_pdl(k2_gateup_mma<TA, kNT>, dim3(grid), dim3(kK2Threads), smem, s, "k2_gateup launch", a);
    } else {
      const size_t smem = (size_t)32 * H + (size_t)kNT * H * sizeof(float) + 2 * (H / 128) * sizeof(float);
      return launch_pdl(k2_gateup<TA, kNT>, dim3(grid), dim3(kK2Threads), smem, s, "k2_gateup launch", a);
    }
  }
  template <typename TA> int run() {
    GateUpArgs<TA> a;
    a.x = (const TA *)x;
    a.w13 = w13; a.s13 = s13; a.sh_w13 = sh_w13; a.sh_s13 = sh_s13; a.sh_gate_w = (const TA *)sh_gate_w;
    a.pf_w2 = pf_w2; a.pf_sh_w2 = sh_w13 ? pf_sh_w2 : nullptr;
    a.pl = plan_view(ws, *L);
    a.sh_w = ws_ptr<float>(ws, L->sh_w);
    a.h = ws_ptr<float>(ws, L->h);
    a.sh_h = ws_ptr<float>(ws, L->sh_h);
    a.T = (int)T; a.H = H; a.I = I; a.Is = sh_w13 ? Is : 0; a.E = E; a.P = (int)T * k;
    a.RG = I / kRows; a.RGs = a.Is / kRows;
    const int max_active = (int)std::min<int64_t>(E, T * k);
    a.routed_ctas = max_active * a.RG;
    const int grid = a.routed_ctas + (sh_w13 ? a.RGs : 0);
    // tokens per pass: up to the MMA's 8 for small calls, 4 beyond (two CTAs per
    // SM); the fp32 path keeps its x staging (kNT * H fp32) within 64 KB
    int cap = sizeof(TA) == 2 ? (T <= 8 ? 8 : 4) : 4;
    if (H > 4096) cap = std::min(cap, 2);
    if (H > 8192) cap = 1;
    switch (tokens_per_pass(T, cap)) {
      case 1: return go<TA, 1>(a, grid);
      case 2: return go<TA, 2>(a, grid);
      case 4: return go<TA, 4>(a, grid);
      default:
        if constexpr (sizeof(TA) == 2) return go<TA, 8>(a, grid);
        else return go<TA, 4>(a, grid);
    }
  }
};

struct DownLaunch {
  int64_t T; int H, I, E, k, Is;
  const void *topk_w; const uint8_t *w2; const float *s2; const uint8_t *sh_w2; const float *sh_s2;
  const void *residual; void *out; void *ws; const WsLayout *L; cudaStream_t s;
  template <typename TA, int kNT> int go(DownArgs<TA> &a, int grid) {
    const int Kmax = std::max(a.I, a.Is);
    const size_t smem = (size_t)a.tile_bytes + (size_t)kNT * Kmax * sizeof(float);
    int rc = launch_pdl(k3_down<TA, kNT>, dim3(grid), dim3(kK3Threads), smem, s, "k3_down launch", a);
    if (rc || a.combine_in_kernel) return rc;
    dim3 g(H / kRows, (unsigned)((T + 15) / 16));
    return launch_pdl(k3_combine<TA>, g, dim3(256), 0, s, "k3_combine launch", a);
  }
  template <typename TA> int run() {
    DownArgs<TA> a;
    a.topk_w = (const TA *)topk_w; a.w2 = w2; a.s2 = s2; a.sh_w2 = sh_w2; a.sh_s2 = sh_s2;
    a.residual = (const TA *)residual; a.out = (TA *)out;
    a.pl = plan_view(ws, *L);
    a.h = ws_ptr<float>(ws, L->h);
    a.sh_h = ws_ptr<float>(ws, L->sh_h);
    a.sh_w = ws_ptr<float>(ws, L->sh_w);
    a.ypart = ws_ptr<float>(ws, L->ypart);
    a.k3_cnt = ws_ptr<int>(ws, L->k3_cnt);
    a.T = (int)T; a.H = H; a.I = I; a.Is = sh_w2 ? Is : 0; a.E = E; a.k = k; a.P = (int)T * k;
    a.RGo = H / kRows;
    a.has_shared = sh_w2 ? 1 : 0;
    const int max_active = (int)std::min<int64_t>(E, T * k);
    a.combine_in_kernel = T <= kCombineInKernelMaxT ? 1 : 0;
    a.tile_bytes = kRows * std::max(I, a.Is);
    if (T == 1 && max_active + a.has_shared <= kK3T1MaxExperts && k <= 32 &&
        std::max(I, a.Is) <= 128 * kK3T1MaxKB) {
      size_t smem = (size_t)max_active * kRows * I + (size_t)kRows * a.Is + ((size_t)k * I + a.Is) * sizeof(float);
      if constexpr (sizeof(TA) == 2) {
        const size_t smem8 = smem + (size_t)(max_active + a.has_shared) * 3 * (std::max(I, a.Is) + 16);
        if (smem8 <= 200 * 1024)
          return launch_pdl(k3_down_t1_f8<TA>, dim3(a.RGo), dim3(kK3F8Threads), smem8, s,
                            "k3_down_t1 launch", a);
        smem += (size_t)(max_active + a.has_shared) * (std::max(I, a.Is) + 8) * 2;
        if (smem <= 200 * 1024)
          return launch_pdl(k3_down_t1_mma<TA>, dim3(a.RGo), dim3(kK3T1Threads), smem, s,
                            "k3_down_t1 launch", a);
      } else {
        if (smem <= 200 * 1024)
          return launch_pdl(k3_down_t1<TA>, dim3(a.RGo), dim3(kK3T1Threads), smem, s, "k3_down_t1 launch", a);
      }
    }
    a.routed_ctas = max_active * a.RGo;
    const int grid = a.routed_ctas + (sh_w2 ? a.RGo : 0);
    switch (tokens_per_pass(T, 8)) {
      case 1: return go<TA, 1>(a, grid);
      case 2: return go<TA, 2>(a, grid);
      case 4: return go<TA, 4>(a, grid);
      default: return go<TA, 8>(a, grid);
    }
  }
};

}  // namespace tmoe

using namespace tmoe;

namespace tmoe {
// L2 prefetch of whole experts' packed weights (cp.async.bulk.prefetch.L2):
// block (c, j) covers chunk c of expert ids[j]; each of its threads issues
// one bulk prefetch of kPfPiece bytes.  No data moves into the SM, nothing is
// waited on; ids outside [0, E) are skipped.
constexpr int kPrefetchThreads = 4;
constexpr int64_t kPrefetchPiece = 16384;
constexpr int64_t kPrefetchChunk = kPrefetchThreads * kPrefetchPiece;
__global__ void __launch_bounds__(kPrefetchThreads) k_prefetch_experts_l2(const uint8_t *w, int64_t expert_bytes,
                                                                          const int64_t *ids, int E) {
  const int64_t e = __ldg(ids + blockIdx.y);
  if (e < 0 || e >= E) return;
  const int64_t off = (int64_t)blockIdx.x * kPrefetchChunk + (int64_t)threadIdx.x * kPrefetchPiece;
  if (off >= expert_bytes) return;
  const uint32_t n = (uint32_t)min(kPrefetchPiece, expert_bytes - off);
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(w + e * expert_bytes + off), "r"(n) : "memory");
}
}  // namespace tmoe

extern "C" int tm_prefetch_experts_l2(const uint8_t *weights, int64_t expert_bytes, int n_experts,
                                      const int64_t *expert_ids, int n_ids, void *stream) {
  TM_REQUIRE(weights && expert_ids, "null pointer");
  TM_REQUIRE(n_experts > 0 && n_ids > 0 && n_ids <= 65535, "bad expert counts (%d experts, %d ids)", n_experts, n_ids);
  TM_REQUIRE(expert_bytes > 0 && expert_bytes % 16 == 0, "expert_bytes (%lld) must be a positive multiple of 16",
             (long long)expert_bytes);
  TM_REQUIRE(reinterpret_cast<uintptr_t>(weights) % 16 == 0, "weights must be 16-byte aligned");
  const int64_t chunks = (expert_bytes + tmoe::kPrefetchChunk - 1) / tmoe::kPrefetchChunk;
  TM_REQUIRE(chunks <= 0x7fffffff, "expert too large");
  tmoe::k_prefetch_experts_l2<<<dim3((unsigned)chunks, (unsigned)n_ids), tmoe::kPrefetchThreads, 0,
                                tmoe::as_stream(stream)>>>(weights, expert_bytes, expert_ids, n_experts);
  return tmoe::cuda_check(cudaGetLastError(), "k_prefetch_experts_l2 launch");
}

extern "C" int tm_moe_decode_gateup(const void *x, int64_t tokens, int hidden, int inter,
                                    int n_experts, int top_k, int act_dtype, const uint8_t *w13,
                                    const float *s13, const uint8_t *sh_w13, const float *sh_s13,
                                    int shared_inter, const void *sh_gate_w, void *ws,
                                    int64_t ws_bytes, void *stream) {
  TM_REQUIRE(x && w13 && s13, "null pointer");
  TM_REQUIRE(hidden % 512 == 0, "hidden (%d) must be a multiple of 512", hidden);
  TM_REQUIRE(inter % 128 == 0 && inter > 0, "inter (%d) must be a positive multiple of 128", inter);
  TM_REQUIRE(!sh_w13 || (sh_s13 && sh_gate_w && shared_inter > 0 && shared_inter % 128 == 0),
             "shared expert needs sh_s13, sh_gate_w and shared_inter %% 128 == 0");
  TM_REQUIRE(aligned(x, 16) && aligned(w13, 16) && (!sh_w13 || aligned(sh_w13, 16)),
             "x and weights must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, inter, sh_w13 ? shared_inter : 0, &L);
  if (rc) return rc;
  GateUpLaunch f{x, tokens, hidden, inter, n_experts, top_k, shared_inter, w13, s13, sh_w13, sh_s13,
                 sh_gate_w, ws, &L, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_moe_decode_gateup_prefetch(const void *x, int64_t tokens, int hidden, int inter,
                                             int n_experts, int top_k, int act_dtype, const uint8_t *w13,
                                             const float *s13, const uint8_t *sh_w13, const float *sh_s13,
                                             int shared_inter, const void *sh_gate_w, const uint8_t *w2,
                                             const uint8_t *sh_w2, void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(x && w13 && s13 && w2, "null pointer");
  TM_REQUIRE(hidden % 512 == 0, "hidden (%d) must be a multiple of 512", hidden);
  TM_REQUIRE(inter % 128 == 0 && inter > 0, "inter (%d) must be a positive multiple of 128", inter);
  TM_REQUIRE(!sh_w13 || (sh_s13 && sh_gate_w && sh_w2 && shared_inter > 0 && shared_inter % 128 == 0),
             "shared expert needs sh_s13, sh_gate_w, sh_w2 and shared_inter %% 128 == 0");
  TM_REQUIRE(aligned(x, 16) && aligned(w13, 16) && aligned(w2, 16) &&
                 (!sh_w13 || (aligned(sh_w13, 16) && aligned(sh_w2, 16))),
             "x and weights must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, inter, sh_w13 ? shared_inter : 0, &L);
  if (rc) return rc;
  GateUpLaunch f{x, tokens, hidden, inter, n_experts, top_k, shared_inter, w13, s13, sh_w13, sh_s13,
                 sh_gate_w, ws, &L, as_stream(stream), w2, sh_w2};
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_moe_decode_down_combine(int64_t tokens, int hidden, int inter, int n_experts,
                                          int top_k, int act_dtype, const void *topk_w,
                                          const uint8_t *w2, const float *s2, const uint8_t *sh_w2,
                                          const float *sh_s2, int shared_inter, const void *residual,
                                          void *out, void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(topk_w && w2 && s2 && out, "null pointer");
  TM_REQUIRE(hidden % 512 == 0, "hidden (%d) must be a multiple of 512", hidden);
  TM_REQUIRE(inter % 128 == 0 && inter > 0, "inter (%d) must be a positive multiple of 128", inter);
  TM_REQUIRE(!sh_w2 || (sh_s2 && shared_inter > 0 && shared_inter % 128 == 0),
             "shared expert needs sh_s2 and shared_inter %% 128 == 0");
  TM_REQUIRE(aligned(w2, 16) && (!sh_w2 || aligned(sh_w2, 16)), "weights must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, inter, sh_w2 ? shared_inter : 0, &L);
  if (rc) return rc;
  DownLaunch f{tokens, hidden, inter, n_experts, top_k, shared_inter, topk_w, w2, s2, sh_w2, sh_s2,
               residual, out, ws, &L, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

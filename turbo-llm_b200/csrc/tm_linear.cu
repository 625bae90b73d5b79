// Dense FP8 block-scaled linear: y = x W^T (+ residual) for the attention and
// other projections of an FP8 checkpoint, without materialising W in the act
// dtype.
//
// Reference: the q/k/v/o projections of execution/layouts/qwen3.py:6-17 are
// loaded by ExpertLoader.load_weight (loader/expert_loader.py:89-114), which
// dequantises W to the act dtype (loader/expert_loader.py:109-112, the same
// arithmetic as dequantize_weight :150-160), and applied with F.linear.
//
// Layout: W [N, K] e4m3 packed like one expert's down projection,
// [N/16][K/16][16 rows][16 B] (each 16x16 chunk one m16k16 MMA A tile, a
// 16-row group one contiguous 16*K-byte tile); scales are the checkpoint's
// weight_scale_inv [N/128][K/128] unchanged.
//
// k6_linear: CTA = 16 output rows.  Its weight tile arrives by four TMA bulk
// copies (one quarter of K per warp) issued before griddepcontrol.wait (W does
// not depend on the previous kernel).  Tokens are taken 8 at a time (the MMA's
// N): their rows are copied in by TMA, scaled by an exact per-token power of 2
// into f16 (exact for bf16/fp16 values) and multiplied on mma.sync m16n8k16
// (e4m3 -> f16 exact, fp32 accumulation, block scale per 128 columns); the
// four warps' K partial sums are added in warp order and rounded once to the
// act dtype.  HBM-bound for decode-sized calls (one pass over W).  One-token
// calls with K % 2048 == 0 take k6_linear_t1_f8 (FP8 MMAs, no conversion).
#include "tm_common.cuh"

namespace tmoe {

constexpr int kLinWarps = 4;
constexpr int kLinThreads = kLinWarps * 32;
constexpr int kLinNT = 8;     // tokens per MMA pass
constexpr int kLinRows = 16;  // output rows per CTA

template <typename TA> struct LinArgs {
  const TA *x;
  const uint8_t *w;
  const float *s;
  const TA *residual;
  TA *out;
  uint32_t *status;  // optional TM_STATUS_* word
  int T, K, N;
  const TA *norm_w;  // k6_linear_t1_f8 only (NULL: none): RMSNorm of x with this weight first
  float eps;
};

template <typename TA>
__global__ void __launch_bounds__(kLinThreads) k6_linear(LinArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  extern __shared__ __align__(128) uint8_t lin_smem[];
  const int tile_bytes = kLinRows * a.K;
  const int quarter = tile_bytes / kLinWarps;
  const int xstride = a.K + 8;  // f16 per staged token row (+16 bytes: no bank conflicts)
  uint8_t *wtile = lin_smem;
  __half *xs = reinterpret_cast<__half *>(lin_smem + tile_bytes);  // [kLinNT][xstride]
  const TA *xraw = reinterpret_cast<const TA *>(xs);
  float *ssc = reinterpret_cast<float *>(lin_smem + tile_bytes + (size_t)kLinNT * xstride * 2);  // [K/128]
  __shared__ float red[kLinWarps][kLinRows][kLinNT];
  __shared__ float xmax[kLinWarps][kLinNT];
  __shared__ int s_shift[kLinNT];
  __shared__ __align__(8) uint64_t bar[kLinWarps];
  __shared__ __align__(8) uint64_t xbar;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int rg = blockIdx.x;
  const int KB = a.K / 128;
  if (tid == 0) {
    for (int q = 0; q < kLinWarps; ++q) mbar_init(&bar[q], 1);
    mbar_init(&xbar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0) {
    const uint8_t *src = a.w + (int64_t)rg * tile_bytes;
    for (int q = 0; q < kLinWarps; ++q) {
      mbar_arrive_expect_tx(&bar[q], quarter);
      tma_bulk_g2s_hint(wtile + q * quarter, src + q * quarter, quarter, &bar[q], l2_evict_first());
    }
  }
  for (int i = tid; i < KB; i += kLinThreads) ssc[i] = __ldg(a.s + (int64_t)((rg * kLinRows) / 128) * KB + i);
  pdl_trigger();
  pdl_wait();  // x (and the residual) come from earlier kernels
  const int cpw = (a.K / 16) / kLinWarps;  // 16-column chunks per warp (multiple of 8: K % 512 == 0)
  const int kc0 = w * cpw;
  const int g = lane >> 2, t = lane & 3;
  const uint32_t wsm = smem_u32(wtile) + (lane & 15) * 16;
  bool first = true;
  for (int tg = 0, grp = 0; tg < a.T; tg += kLinNT, ++grp) {
    const int nt = min(kLinNT, a.T - tg);
    if (tg) __syncthreads();  // everyone is done with the previous group's rows
    if (tid == 0) {
      fence_proxy_async();
      const uint32_t rowb = (uint32_t)a.K * sizeof(TA);
      mbar_arrive_expect_tx(&xbar, nt * rowb);
      for (int j = 0; j < nt; ++j) tma_bulk_g2s(xs + (size_t)j * xstride, a.x + (int64_t)(tg + j) * a.K, rowb, &xbar);
    }
    const bool xok = mbar_wait_bounded(&xbar, grp & 1);
    if (__syncthreads_or(!xok)) {
      if (tid == 0) {
        if (a.status) atomicOr(a.status, TM_STATUS_TIMEOUT);
        mbar_wait_bounded(&xbar, grp & 1);
        for (int q = 0; q < kLinWarps; ++q) mbar_wait_bounded(&bar[q], 0);
      }
      return;
    }
    // per-token max |x| over this warp's quarter of K -> exact power-of-2 shift
    for (int j = 0; j < nt; ++j) {
      float m = 0.f;
      const int c_lo = w * (a.K / kLinWarps), c_hi = c_lo + a.K / kLinWarps;
      for (int c = c_lo + lane; c < c_hi; c += 32) m = fmaxf(m, fabsf(Act<TA>::to_f(xraw[(size_t)j * xstride + c])));
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
      if (lane == 0) xmax[w][j] = m;
    }
    __syncthreads();
    if (tid < nt) {
      float m = 0.f;
#pragma unroll
      for (int ww = 0; ww < kLinWarps; ++ww) m = fmaxf(m, xmax[ww][tid]);
      s_shift[tid] = f16_shift(m);
    }
    __syncthreads();
    for (int i = tid; i < nt * (a.K / 2); i += kLinThreads) {  // in place: each pair read then written by one thread
      const int j = i / (a.K / 2), c = (i % (a.K / 2)) * 2;
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
          if (a.status) atomicOr(a.status, TM_STATUS_TIMEOUT);
          for (int q = 0; q < kLinWarps; ++q) mbar_wait_bounded(&bar[q], 0);
        }
        return;
      }
    }
    const __half *xrow = xs + (size_t)min(g, nt - 1) * xstride + 4 * t;  // B column n = g
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int blk = 0; blk < cpw / 8; ++blk) {
      float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f};  // two independent MMA chains
#pragma unroll
      for (int i = 0; i < 8; i += 2) {
        const int kc = kc0 + blk * 8 + i;
        uint32_t r0, r1, r2, r3, a0, a1, a2, a3, c0, c1, c2, c3;
        ldsm_x2(wsm + kc * 256, r0, r1);
        ldsm_x2(wsm + (kc + 1) * 256, r2, r3);
        const uint2 bx0 = *reinterpret_cast<const uint2 *>(xrow + kc * 16);
        const uint2 bx1 = *reinterpret_cast<const uint2 *>(xrow + (kc + 1) * 16);
        e4m3x4_to_f16x2x2(r0, a0, a2);
        e4m3x4_to_f16x2x2(r1, a1, a3);
        e4m3x4_to_f16x2x2(r2, c0, c2);
        e4m3x4_to_f16x2x2(r3, c1, c3);
        mma_16816(d0, a0, a1, a2, a3, bx0.x, bx0.y);
        mma_16816(d1, c0, c1, c2, c3, bx1.x, bx1.y);
      }
      const float sblk = ssc[(kc0 + blk * 8) / 8];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = fmaf(d0[q] + d1[q], sblk, acc[q]);
    }
    // D fragment: (row g, tokens 2t, 2t+1), (row g+8, tokens 2t, 2t+1)
    red[w][g][2 * t] = acc[0];
    red[w][g][2 * t + 1] = acc[1];
    red[w][g + 8][2 * t] = acc[2];
    red[w][g + 8][2 * t + 1] = acc[3];
    __syncthreads();
    if (tid < nt * kLinRows) {
      const int j = tid / kLinRows, r = tid % kLinRows;
      float y = 0.f;
#pragma unroll
      for (int ww = 0; ww < kLinWarps; ++ww) y += red[ww][r][j];
      y *= ldexpf(1.0f, s_shift[j]);
      const int64_t o = (int64_t)(tg + j) * a.N + rg * kLinRows + r;
      if (a.residual) y += Act<TA>::to_f(Act<TA>::ld_cg(a.residual + o));
      a.out[o] = Act<TA>::from_f(y);
    }
  }
}

// One token, 16-bit activations (the decode step's projections): the token
// enters FP8 mma.sync m16n8k32 as three e4m3 terms x * 2^s ~= hi + mid/16 +
// lo/256 (one MMA column each, rows 16 bytes apart in bank order; the same
// split as the one-token expert kernels), the packed e4m3 tile is multiplied
// as it is (no e4m3 -> f16 conversion).  kW warps split K; each warp waits
// only for its own part of the tile and holds its kSt B fragment pairs in
// registers; four independent MMA chains, block scale per 128 columns; the
// warps' partial sums are added in warp order and rounded once to the act
// dtype.
template <typename TA, int kW, int kSt>
__global__ void __launch_bounds__(kW * 32) k6_linear_t1_f8(LinArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  extern __shared__ __align__(128) uint8_t lin_smem[];
  const int tile_bytes = kLinRows * a.K;
  const int part = tile_bytes / kW;
  const int XS = a.K + 16;
  uint8_t *wtile = lin_smem;
  uint8_t *xb = lin_smem + tile_bytes;                          // [3][XS] e4m3: hi, mid, lo
  const TA *xraw = reinterpret_cast<const TA *>(xb + XS);       // [K] act (before the split)
  float *ssc = reinterpret_cast<float *>(xb + 3 * XS);          // [K/128]
  __shared__ float red[kW][kLinRows];
  __shared__ float xmax[kW];
  __shared__ float nred[kW];
  __shared__ int s_shift;
  __shared__ __align__(8) uint64_t bar[kW];
  __shared__ __align__(8) uint64_t xbar;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int rg = blockIdx.x;
  const int KB = a.K / 128;
  if (tid == 0) {
    for (int q = 0; q < kW; ++q) mbar_init(&bar[q], 1);
    mbar_init(&xbar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  if (tid == 0) {  // W does not depend on the previous kernel: stream it now
    const uint8_t *src = a.w + (int64_t)rg * tile_bytes;
    for (int q = 0; q < kW; ++q) {
      mbar_arrive_expect_tx(&bar[q], part);
      tma_bulk_g2s_hint(wtile + q * part, src + q * part, part, &bar[q], l2_evict_first());
    }
  }
  for (int i = tid; i < KB; i += kW * 32) ssc[i] = __ldg(a.s + (int64_t)((rg * kLinRows) / 128) * KB + i);
  // RMSNorm weights (they do not depend on the previous kernel): thread tid
  // owns elements (c * 256 + tid) * 4 .. + 3, c < 4, as k8_rmsnorm does
  const bool norm = a.norm_w != nullptr;
  float wv[4][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = (c * 256 + tid) * 4 + e;
      wv[c][e] = (norm && i < a.K) ? Act<TA>::to_f(a.norm_w[i]) : 0.f;
    }
  pdl_trigger();
  pdl_wait();  // x (and the residual) come from earlier kernels
  if (tid == 0) {
    const uint32_t rowb = (uint32_t)a.K * sizeof(TA);
    mbar_arrive_expect_tx(&xbar, rowb);
    tma_bulk_g2s(const_cast<TA *>(xraw), a.x, rowb, &xbar);
  }
  const bool xok = mbar_wait_bounded(&xbar, 0);
  if (__syncthreads_or(!xok)) {
    if (tid == 0) {
      if (a.status) atomicOr(a.status, TM_STATUS_TIMEOUT);
      mbar_wait_bounded(&xbar, 0);
      for (int q = 0; q < kW; ++q) mbar_wait_bounded(&bar[q], 0);
    }
    return;
  }
  if (norm) {
    // Qwen3MoeRMSNorm of the token with k8_rmsnorm's arithmetic and thread
    // decomposition (8 warps of 256 threads, the same sums in the same order:
    // the same bits), kept in registers; then max |y| and the split of y
    float v[4][4];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = (c * 256 + tid) * 4;
#pragma unroll
      for (int e = 0; e < 4; ++e) v[c][e] = 0.f;
      if (i < a.K) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[c][e] = Act<TA>::to_f(xraw[i + e]);
          ss = fmaf(v[c][e], v[c][e], ss);
        }
      }
    }
    ss = warp_sum(ss);
    if (lane == 0) nred[w] = ss;
    __syncthreads();  // (also: every thread has read its raw x, which the split overwrites)
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kW; ++i) tot += nred[i];
    const float r = rsqrtf(tot / (float)a.K + a.eps);
    float m = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        v[c][e] = Act<TA>::round(Act<TA>::round(v[c][e] * r) * wv[c][e]);
        m = fmaxf(m, fabsf(v[c][e]));
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) xmax[w] = m;
    __syncthreads();
    if (tid == 0) {
      float mm = 0.f;
#pragma unroll
      for (int ww = 0; ww < kW; ++ww) mm = fmaxf(mm, xmax[ww]);
      s_shift = e4m3_shift(mm);
    }
    __syncthreads();
    const float sc = ldexpf(1.0f, s_shift);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = (c * 256 + tid) * 4;
      if (i < a.K) {
        float q[4] = {v[c][0] * sc, v[c][1] * sc, v[c][2] * sc, v[c][3] * sc};
        uint32_t h, md, l;
        e4m3_split3(q, h, md, l);
        *reinterpret_cast<uint32_t *>(xb + i) = h;
        *reinterpret_cast<uint32_t *>(xb + XS + i) = md;
        *reinterpret_cast<uint32_t *>(xb + 2 * XS + i) = l;
      }
    }
  } else {
  {  // max |x| -> power-of-2 scale
    float m = 0.f;
    const int c_lo = w * (a.K / kW), c_hi = c_lo + a.K / kW;
    for (int c = c_lo + lane; c < c_hi; c += 32) m = fmaxf(m, fabsf(Act<TA>::to_f(xraw[c])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) xmax[w] = m;
  }
  __syncthreads();
  if (tid == 0) {
    float m = 0.f;
#pragma unroll
    for (int ww = 0; ww < kW; ++ww) m = fmaxf(m, xmax[ww]);
    s_shift = e4m3_shift(m);
  }
  __syncthreads();
  {  // split: every thread first reads its elements (the raw row overlaps mid/lo)
    constexpr int kMaxSteps = 6;  // K <= 6144 at 256 threads
    const int steps = a.K / (4 * kW * 32);
    const float sc = ldexpf(1.0f, s_shift);
    float v[kMaxSteps][4];
#pragma unroll
    for (int k = 0; k < kMaxSteps; ++k)
      if (k < steps) {
        const int c = 4 * (tid + k * kW * 32);
#pragma unroll
        for (int u = 0; u < 4; ++u) v[k][u] = Act<TA>::to_f(xraw[c + u]) * sc;
      }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kMaxSteps; ++k)
      if (k < steps) {
        const int c = 4 * (tid + k * kW * 32);
        uint32_t h, md, l;
        e4m3_split3(v[k], h, md, l);
        *reinterpret_cast<uint32_t *>(xb + c) = h;
        *reinterpret_cast<uint32_t *>(xb + XS + c) = md;
        *reinterpret_cast<uint32_t *>(xb + 2 * XS + c) = l;
      }
  }
  }
  __syncthreads();
  const int cpw = (a.K / 16) / kW;  // 16-column chunks per warp (== 2 * kSt)
  const int kc0 = w * cpw;
  const int g = lane >> 2, t = lane & 3;
  // B column n = g: 0 hi, 1 mid, 2 lo (columns 3-7 repeat lo and are not read)
  const uint8_t *xsel = xb + min(g, 2) * XS + kc0 * 16 + 4 * t;
  uint32_t bx[kSt][2];
#pragma unroll
  for (int st = 0; st < kSt; ++st) {
    bx[st][0] = *reinterpret_cast<const uint32_t *>(xsel + st * 32);
    bx[st][1] = *reinterpret_cast<const uint32_t *>(xsel + st * 32 + 16);
  }
  const bool part_ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bar[w], 0));
  // A (ldmatrix.x4): lanes 0-15 rows 0-15 of chunk kc, lanes 16-31 of chunk kc+1
  const uint32_t wsm = smem_u32(wtile) + (kc0 + (lane >> 4)) * 256 + (lane & 15) * 16;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (part_ok) {
#pragma unroll
    for (int blk = 0; blk < kSt / 4; ++blk) {
      float d[4][4];  // four independent MMA chains, one 32-column step each
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int q = 0; q < 4; ++q) d[c][q] = 0.f;
#pragma unroll
      for (int st = 0; st < 4; ++st) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(wsm + (blk * 8 + 2 * st) * 256, a0, a1, a2, a3);
        mma_16832_e4m3(d[st], a0, a1, a2, a3, bx[blk * 4 + st][0], bx[blk * 4 + st][1]);
      }
      const float sblk = ssc[(kc0 + blk * 8) / 8];
#pragma unroll
      for (int q = 0; q < 4; ++q) acc[q] = fmaf((d[0][q] + d[1][q]) + (d[2][q] + d[3][q]), sblk, acc[q]);
    }
  }
  // D: lane (g, t=0) holds columns hi, mid of rows g, g+8; lane (g, t=1) lo
  const float lo0 = __shfl_down_sync(0xffffffffu, acc[0], 1), lo8 = __shfl_down_sync(0xffffffffu, acc[2], 1);
  if (t == 0) {
    red[w][g] = acc[0] + (acc[1] + lo0 * 0.0625f) * 0.0625f;
    red[w][g + 8] = acc[2] + (acc[3] + lo8 * 0.0625f) * 0.0625f;
  }
  if (__syncthreads_or(!part_ok)) {  // a part never landed: flag, let the copies finish, no output
    if (tid == 0) {
      if (a.status) atomicOr(a.status, TM_STATUS_TIMEOUT);
      for (int q = 0; q < kW; ++q) mbar_wait_bounded(&bar[q], 0);
    }
    return;
  }
  if (tid < kLinRows) {
    float y = 0.f;
#pragma unroll
    for (int ww = 0; ww < kW; ++ww) y += red[ww][tid];
    y *= ldexpf(1.0f, -s_shift);
    const int64_t o = (int64_t)rg * kLinRows + tid;
    if (a.residual) y += Act<TA>::to_f(Act<TA>::ld_cg(a.residual + o));
    a.out[o] = Act<TA>::from_f(y);
  }
}

// fp32 activations: a CUDA-core kernel on the same packed layout.  Every
// weight is dequantised as the reference's fp32 load_weight does (e4m3 ->
// fp32 exactly, times its block scale: one fp32 rounding) and accumulated in
// fp32: the reference's fp32 F.linear up to the order of the sums.  CTA = one
// packed 16-row group; warp w takes rows 4w..4w+3, lane j the 16-column
// chunks j, j + 32, ... of a row; the lanes' sums are added by shuffles.
__global__ void __launch_bounds__(kLinThreads) k6_linear_f32(LinArgs<float> a) {
  pdl_wait();
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int rg = blockIdx.x;
  const int KC = a.K / 16, KB = a.K / 128;
  const uint8_t *tile = a.w + (int64_t)rg * kLinRows * a.K;   // [K/16][16 rows][16 B]
  for (int rr = 0; rr < kLinRows / kLinWarps; ++rr) {
    const int r = w * (kLinRows / kLinWarps) + rr;
    const int n = rg * kLinRows + r;
    const float *srow = a.s + (int64_t)(n / 128) * KB;
    for (int t = 0; t < a.T; ++t) {
      const float *xt = a.x + (int64_t)t * a.K;
      float acc = 0.f;
      for (int kc = lane; kc < KC; kc += 32) {
        const uint4 raw = *reinterpret_cast<const uint4 *>(tile + ((int64_t)kc * kLinRows + r) * 16);
        const float sc = srow[kc / 8];
        const uint32_t wd[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          float f[4];
          e4m3x4_to_f32(wd[q], f[0], f[1], f[2], f[3]);
#pragma unroll
          for (int i = 0; i < 4; ++i) acc = fmaf(__ldcg(xt + kc * 16 + q * 4 + i), f[i] * sc, acc);
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        const int64_t o = (int64_t)t * a.N + n;
        a.out[o] = a.residual ? acc + __ldcg(a.residual + o) : acc;
      }
    }
  }
}

static size_t linear_smem(int K) {
  return (size_t)kLinRows * K + (size_t)kLinNT * (K + 8) * 2 + (size_t)(K / 128) * sizeof(float);
}

struct LinearLaunch {
  const void *x; int64_t T; int K, N;
  const uint8_t *w; const float *s; const void *residual; void *out; uint32_t *status; cudaStream_t st;
  const void *norm_w = nullptr; float eps = 0.f;   // one-token FP8 path only
  template <typename TA, int kSt> int launch_t1(const LinArgs<TA> &a, size_t smem) {
    int rc = ensure_smem(reinterpret_cast<const void *>(k6_linear_t1_f8<TA, 8, kSt>), smem);
    if (rc) return rc;
    return launch_pdl(k6_linear_t1_f8<TA, 8, kSt>, dim3(N / kLinRows), dim3(8 * 32), smem, st,
                      "k6_linear_t1_f8 launch", a);
  }
  template <typename TA> int run() {
    if constexpr (sizeof(TA) != 2) {
      LinArgs<float> a;
      a.x = (const float *)x; a.w = w; a.s = s; a.residual = (const float *)residual; a.out = (float *)out;
      a.status = status; a.T = (int)T; a.K = K; a.N = N;
      a.norm_w = nullptr; a.eps = 0.f;
      return launch_pdl(k6_linear_f32, dim3(N / kLinRows), dim3(kLinThreads), 0, st, "k6_linear_f32 launch", a);
    } else {
      LinArgs<TA> a;
      a.x = (const TA *)x; a.w = w; a.s = s; a.residual = (const TA *)residual; a.out = (TA *)out;
      a.status = status; a.T = (int)T; a.K = K; a.N = N;
      a.norm_w = (const TA *)norm_w; a.eps = eps;
      if (T == 1 && K % 2048 == 0 && K <= 6144) {  // one token: FP8 MMAs on the split activation, 8 warps
        const size_t smem1 = (size_t)kLinRows * K + (size_t)3 * (K + 16) + (size_t)(K / 128) * sizeof(float);
        switch (K) {  // kSt = 32-column MMA steps per warp = K / 256
          case 2048: return launch_t1<TA, 8>(a, smem1);
          case 4096: return launch_t1<TA, 16>(a, smem1);
          default: return launch_t1<TA, 24>(a, smem1);
        }
      }
      const size_t smem = linear_smem(K);
      int rc = ensure_smem(reinterpret_cast<const void *>(k6_linear<TA>), smem);
      if (rc) return rc;
      return launch_pdl(k6_linear<TA>, dim3(N / kLinRows), dim3(kLinThreads), smem, st, "k6_linear launch", a);
    }
  }
};

}  // namespace tmoe

using namespace tmoe;

extern "C" int tm_fp8_linear(const void *x, int64_t tokens, int in_features, int out_features, int act_dtype,
                             const uint8_t *w_packed, const float *scale_inv, const void *residual, void *out,
                             uint32_t *status, void *stream) {
  TM_REQUIRE(x && w_packed && scale_inv && out, "null pointer");
  TM_REQUIRE(tokens >= 1 && tokens <= (1 << 20), "tokens %lld out of range", (long long)tokens);
  TM_REQUIRE(in_features % 512 == 0 && in_features > 0 && in_features <= 6144,
             "in_features %d must be a positive multiple of 512, at most 6144", in_features);
  TM_REQUIRE(out_features % 128 == 0 && out_features > 0, "out_features %d must be a positive multiple of 128",
             out_features);
  TM_REQUIRE(aligned(x, 16) && aligned(w_packed, 16) && aligned(out, 16) && (!residual || aligned(residual, 2)),
             "x, w_packed and out must be 16-byte aligned");
  LinearLaunch f{x, tokens, in_features, out_features, w_packed, scale_inv, residual, out, status,
                 as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_rmsnorm_fp8_linear(const void *x, int hidden, int act_dtype, const void *norm_w, float eps,
                                     int out_features, const uint8_t *w_packed, const float *scale_inv,
                                     const void *residual, void *out, uint32_t *status, void *stream) {
  TM_REQUIRE(x && norm_w && w_packed && scale_inv && out, "null pointer");
  TM_REQUIRE(act_dtype == TM_DTYPE_BF16 || act_dtype == TM_DTYPE_F16, "16-bit activations only");
  TM_REQUIRE(hidden == 2048 || hidden == 4096, "hidden %d unsupported (2048 or 4096)", hidden);
  TM_REQUIRE(out_features % 128 == 0 && out_features > 0, "out_features %d must be a positive multiple of 128",
             out_features);
  TM_REQUIRE(aligned(x, 16) && aligned(w_packed, 16) && aligned(out, 16) && aligned(norm_w, 2) &&
                 (!residual || aligned(residual, 2)),
             "x, w_packed and out must be 16-byte aligned");
  LinearLaunch f{x, 1, hidden, out_features, w_packed, scale_inv, residual, out, status, as_stream(stream)};
  f.norm_w = norm_w;
  f.eps = eps;
  return dispatch_act(act_dtype, f);
}

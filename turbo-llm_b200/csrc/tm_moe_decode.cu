// K2 (gate+up dequant-GEMV + SwiGLU) and K3 (down dequant-GEMV + routing-
// weighted combine) for the decode path (1..64 tokens per layer call).
//
// Reference: moe_seq (execution/moe.py:7-20), the multi-token loop of
// MoEExecutor.execute_layer (moe.py:157-180) and the shared expert
// (moe.py:73-85, 191-202).  Weights stream from the packed layout of
// tm_pack_experts; every lane owns one weight row and reads 16 bytes per
// column chunk, so a warp reads 512 contiguous bytes per instruction.  The
// activations a lane needs are the same for all lanes (same columns), so they
// come from shared memory as broadcasts.  Block scales are uniform per warp
// (32 rows and 128 columns sit inside one 128x128 block).
#include "tm_common.cuh"

namespace tmoe {

constexpr int kK2Warps = 4;       // K2: 4 warps x 128 columns = 512 columns per CTA
constexpr int kK2Threads = kK2Warps * 32;
constexpr int kK3Threads = 64;    // K3: 2 warps, one per half of the reduction dimension
constexpr int kCombineInKernelMaxT = 64;

struct PlanView {
  const int *meta, *counts, *offsets, *act_list, *slot_token, *pair_slot;
};

static PlanView plan_view(void *ws, const WsLayout &L) {
  return PlanView{ws_ptr<int>(ws, L.meta),     ws_ptr<int>(ws, L.counts),
                  ws_ptr<int>(ws, L.offsets),  ws_ptr<int>(ws, L.act_list),
                  ws_ptr<int>(ws, L.slot_token), ws_ptr<int>(ws, L.pair_slot)};
}

// Accumulate 16 weights (one 16-byte chunk) times 16 broadcast activations.
__device__ __forceinline__ float dot16(const float (&w)[16], const float *xr) {
  const float4 a = *reinterpret_cast<const float4 *>(xr);
  const float4 b = *reinterpret_cast<const float4 *>(xr + 4);
  const float4 c = *reinterpret_cast<const float4 *>(xr + 8);
  const float4 d = *reinterpret_cast<const float4 *>(xr + 12);
  float s = w[0] * a.x;
  s = fmaf(w[1], a.y, s); s = fmaf(w[2], a.z, s); s = fmaf(w[3], a.w, s);
  s = fmaf(w[4], b.x, s); s = fmaf(w[5], b.y, s); s = fmaf(w[6], b.z, s); s = fmaf(w[7], b.w, s);
  s = fmaf(w[8], c.x, s); s = fmaf(w[9], c.y, s); s = fmaf(w[10], c.z, s); s = fmaf(w[11], c.w, s);
  s = fmaf(w[12], d.x, s); s = fmaf(w[13], d.y, s); s = fmaf(w[14], d.z, s); s = fmaf(w[15], d.w, s);
  return s;
}

__device__ __forceinline__ void decode16(const uint4 &v, float (&w)[16]) {
  e4m3x4_to_f32(v.x, w[0], w[1], w[2], w[3]);
  e4m3x4_to_f32(v.y, w[4], w[5], w[6], w[7]);
  e4m3x4_to_f32(v.z, w[8], w[9], w[10], w[11]);
  e4m3x4_to_f32(v.w, w[12], w[13], w[14], w[15]);
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
  int *k2_cnt;
  float *gu_part, *sh_gu_part, *shg_part, *sh_w, *h, *sh_h;
  int T, H, I, Is, E, P, KQ, RG, RGs;
  int routed_ctas;  // max_active * RG * KQ
};

template <typename TA, int kNT>
__global__ void __launch_bounds__(kK2Threads, 4) k2_gateup(GateUpArgs<TA> a) {
  __shared__ __align__(16) float xs[kNT][512];
  __shared__ float red[kK2Warps][kNT][2][32];
  __shared__ float gred[kK2Warps][kNT];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  int b = blockIdx.x;
  bool shared_expert;
  int aidx, rg, kq, n, slot0, I, RG;
  const uint8_t *wbase;
  const float *sbase;
  if (b < a.routed_ctas) {
    shared_expert = false;
    aidx = b / (a.RG * a.KQ);
    const int rem = b % (a.RG * a.KQ);
    rg = rem / a.KQ;
    kq = rem % a.KQ;
    if (aidx >= a.pl.meta[kMetaNActive]) return;
    const int e = a.pl.act_list[aidx];
    n = a.pl.counts[e];
    slot0 = a.pl.offsets[e];
    I = a.I;
    RG = a.RG;
    wbase = a.w13 + (int64_t)e * 2 * a.I * a.H;
    sbase = a.s13 + (int64_t)e * 2 * (a.I / 128) * (a.H / 128);
  } else {
    shared_expert = true;
    b -= a.routed_ctas;
    aidx = a.E;
    rg = b / a.KQ;
    kq = b % a.KQ;
    n = a.T;
    slot0 = 0;
    I = a.Is;
    RG = a.RGs;
    wbase = a.sh_w13;
    sbase = a.sh_s13;
  }
  const int KC = a.H / 16, HB = a.H / 128;
  const int c0 = kq * 512 + w * 128;  // this warp's 128 columns
  // issue all 16 weight loads of this warp's tile (8 chunks x gate/up)
  uint4 wv[8][2];
  {
    const uint8_t *p = wbase + ((int64_t)rg * KC + c0 / 16) * 1024 + lane * 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wv[i][0] = ldg_stream(p + i * 1024);
      wv[i][1] = ldg_stream(p + i * 1024 + 512);
    }
  }
  const int ib = (rg * 32) / 128;
  const float sg = sbase[(ib * 2 + 0) * HB + c0 / 128];
  const float su = sbase[(ib * 2 + 1) * HB + c0 / 128];
  float *part = shared_expert ? a.sh_gu_part : a.gu_part;
  const int nslots = shared_expert ? a.T : a.P;

  for (int tg = 0; tg < n; tg += kNT) {
    const int nt = min(kNT, n - tg);
    __syncthreads();  // xs / red reuse across groups
    for (int i = tid; i < nt * 512; i += kK2Threads) {
      const int j = i >> 9, c = i & 511;
      const int t = shared_expert ? (tg + j) : a.pl.slot_token[slot0 + tg + j];
      xs[j][c] = Act<TA>::to_f(a.x[(int64_t)t * a.H + kq * 512 + c]);
    }
    __syncthreads();
    float ag[kNT], au[kNT];
#pragma unroll
    for (int j = 0; j < kNT; ++j) { ag[j] = 0.f; au[j] = 0.f; }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t gw[4] = {wv[i][0].x, wv[i][0].y, wv[i][0].z, wv[i][0].w};
      const uint32_t uw[4] = {wv[i][1].x, wv[i][1].y, wv[i][1].z, wv[i][1].w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // 4 columns per 32-bit word
        float g0, g1, g2, g3, u0, u1, u2, u3;
        e4m3x4_to_f32(gw[q], g0, g1, g2, g3);
        e4m3x4_to_f32(uw[q], u0, u1, u2, u3);
#pragma unroll
        for (int j = 0; j < kNT; ++j) {
          if (j < nt) {
            const float4 xv = *reinterpret_cast<const float4 *>(&xs[j][w * 128 + i * 16 + q * 4]);
            ag[j] = fmaf(g0, xv.x, ag[j]); ag[j] = fmaf(g1, xv.y, ag[j]);
            ag[j] = fmaf(g2, xv.z, ag[j]); ag[j] = fmaf(g3, xv.w, ag[j]);
            au[j] = fmaf(u0, xv.x, au[j]); au[j] = fmaf(u1, xv.y, au[j]);
            au[j] = fmaf(u2, xv.z, au[j]); au[j] = fmaf(u3, xv.w, au[j]);
          }
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kNT; ++j) {
      red[w][j][0][lane] = ag[j] * sg;
      red[w][j][1][lane] = au[j] * su;
    }
    if (shared_expert && rg == 0) {
      // partial shared-gate logit over this CTA's 512 columns (moe.py:81-83)
      for (int j = 0; j < nt; ++j) {
        float s = 0.f;
        for (int c = lane; c < 128; c += 32)
          s = fmaf(xs[j][w * 128 + c], Act<TA>::to_f(a.sh_gate_w[c0 + c]), s);
        s = warp_sum(s);
        if (lane == 0) gred[w][j] = s;
      }
    }
    __syncthreads();
    for (int i = tid; i < nt * 64; i += kK2Threads) {
      const int j = i >> 6, mat = (i >> 5) & 1, r = i & 31;
      float s = 0.f;
#pragma unroll
      for (int ww = 0; ww < kK2Warps; ++ww) s += red[ww][j][mat][r];
      part[(((int64_t)kq * nslots + slot0 + tg + j) * 2 + mat) * I + rg * 32 + r] = s;
    }
    if (shared_expert && rg == 0 && tid < nt) {
      float s = 0.f;
#pragma unroll
      for (int ww = 0; ww < kK2Warps; ++ww) s += gred[ww][tid];
      a.shg_part[(int64_t)kq * a.T + tg + tid] = s;
    }
  }
  // the last of the KQ column-quarter CTAs of (expert, row group) finishes
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    int *cnt = a.k2_cnt + aidx * kMaxRG + rg;
    const int prev = atomicAdd(cnt, 1);
    s_last = (prev == a.KQ - 1);
    if (s_last) *cnt = 0;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  float *hout = shared_expert ? a.sh_h : a.h;
  for (int i = tid; i < n * 32; i += kK2Threads) {
    const int j = i >> 5, r = i & 31;
    float g = 0.f, u = 0.f;
    for (int q = 0; q < a.KQ; ++q) {
      g += ld_cg(part + (((int64_t)q * nslots + slot0 + j) * 2 + 0) * I + rg * 32 + r);
      u += ld_cg(part + (((int64_t)q * nslots + slot0 + j) * 2 + 1) * I + rg * 32 + r);
    }
    hout[(int64_t)(slot0 + j) * I + rg * 32 + r] = silu(g) * u;
  }
  if (shared_expert && rg == 0) {
    for (int t = tid; t < a.T; t += kK2Threads) {
      float s = 0.f;
      for (int q = 0; q < a.KQ; ++q) s += ld_cg(a.shg_part + (int64_t)q * a.T + t);
      // F.linear output and torch.sigmoid both produce the act dtype
      const float logit = Act<TA>::round(s);
      a.sh_w[t] = Act<TA>::round(1.0f / (1.0f + __expf(-logit)));
    }
  }
}

// ===================================================================== K3 ====
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
  int routed_ctas;  // max(max_active,1) * RGo
  int has_shared;
  int combine_in_kernel;
};

// out[t, n] for rows [n0, n0 + nrows) and tokens [t0, t1): k-order weighted sum,
// then the gated shared expert, then the residual.
template <typename TA>
__device__ __forceinline__ void combine_rows(const DownArgs<TA> &a, int t0, int t1, int n0, int nrows,
                                             int tid, int nthreads) {
  for (int i = tid; i < (t1 - t0) * nrows; i += nthreads) {
    const int t = t0 + i / nrows, nn = n0 + i % nrows;
    float y = 0.f;
    for (int kk = 0; kk < a.k; ++kk) {
      const int slot = a.pl.pair_slot[(int64_t)t * a.k + kk];
      if (slot >= 0)
        y = fmaf(Act<TA>::to_f(a.topk_w[(int64_t)t * a.k + kk]), ld_cg(a.ypart + (int64_t)slot * a.H + nn), y);
    }
    if (a.has_shared) y = fmaf(ld_cg(a.sh_w + t), ld_cg(a.ypart + (int64_t)(a.P + t) * a.H + nn), y);
    if (a.residual) y += Act<TA>::to_f(a.residual[(int64_t)t * a.H + nn]);
    a.out[(int64_t)t * a.H + nn] = Act<TA>::from_f(y);
  }
}

template <typename TA, int kNT>
__global__ void __launch_bounds__(kK3Threads) k3_down(DownArgs<TA> a) {
  extern __shared__ __align__(16) float hs[];  // [kNT][K]
  __shared__ float red[2][kNT][32];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  int b = blockIdx.x;
  const int n_active = a.pl.meta[kMetaNActive];
  bool shared_expert, idle = false;
  int rgo, n, slot0, K;
  const uint8_t *wbase;
  const float *sbase;
  const float *hsrc;
  if (b < a.routed_ctas) {
    shared_expert = false;
    const int aidx = b / a.RGo;
    rgo = b % a.RGo;
    if (aidx >= max(n_active, 1)) return;
    if (n_active == 0) {
      idle = true;  // no routed pair: still count this CTA so the combine runs
      n = 0; slot0 = 0; K = a.I; wbase = nullptr; sbase = nullptr; hsrc = nullptr;
    } else {
      const int e = a.pl.act_list[aidx];
      n = a.pl.counts[e];
      slot0 = a.pl.offsets[e];
      K = a.I;
      wbase = a.w2 + (int64_t)e * a.H * a.I;
      sbase = a.s2 + (int64_t)e * (a.H / 128) * (a.I / 128);
      hsrc = a.h;
    }
  } else {
    shared_expert = true;
    rgo = b - a.routed_ctas;
    n = a.T;
    slot0 = 0;
    K = a.Is;
    wbase = a.sh_w2;
    sbase = a.sh_s2;
    hsrc = a.sh_h;
  }
  if (!idle) {
    const int KC2 = K / 16, KB = K / 128;
    const int half = KC2 / 2;          // chunks per warp (K % 256 == 0: whole scale blocks)
    const int kc0 = w * half;
    const uint8_t *p = wbase + ((int64_t)rgo * KC2 + kc0) * 512 + lane * 16;
    const float *srow = sbase + (int64_t)((rgo * 32) / 128) * KB;
    const int ypbase = shared_expert ? a.P : 0;
    for (int tg = 0; tg < n; tg += kNT) {
      const int nt = min(kNT, n - tg);
      __syncthreads();
      for (int i = tid; i < nt * K; i += kK3Threads) {
        const int j = i / K, c = i % K;
        hs[j * K + c] = ld_cg(hsrc + (int64_t)(slot0 + tg + j) * K + c);
      }
      __syncthreads();
      float acc[kNT];
#pragma unroll
      for (int j = 0; j < kNT; ++j) acc[j] = 0.f;
      // 8 chunks (= one 128-column scale block) per step, next step's loads in flight
      uint4 cur[8], nxt[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) cur[i] = ldg_stream(p + i * 512);
      for (int blk = 0; blk < half / 8; ++blk) {
        const bool more = (blk + 1) < half / 8;
        if (more) {
#pragma unroll
          for (int i = 0; i < 8; ++i) nxt[i] = ldg_stream(p + ((blk + 1) * 8 + i) * 512);
        }
        float bacc[kNT];
#pragma unroll
        for (int j = 0; j < kNT; ++j) bacc[j] = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float wf[16];
          decode16(cur[i], wf);
#pragma unroll
          for (int j = 0; j < kNT; ++j)
            if (j < nt) bacc[j] += dot16(wf, &hs[j * K + (kc0 + blk * 8 + i) * 16]);
        }
        const float sc = srow[(kc0 + blk * 8) / 8];
#pragma unroll
        for (int j = 0; j < kNT; ++j) acc[j] = fmaf(bacc[j], sc, acc[j]);
        if (more) {
#pragma unroll
          for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
        }
      }
#pragma unroll
      for (int j = 0; j < kNT; ++j) red[w][j][lane] = acc[j];
      __syncthreads();
      for (int i = tid; i < nt * 32; i += kK3Threads) {
        const int j = i >> 5, r = i & 31;
        a.ypart[(int64_t)(ypbase + slot0 + tg + j) * a.H + rgo * 32 + r] = red[0][j][r] + red[1][j][r];
      }
    }
  }
  if (!a.combine_in_kernel) return;
  // the last CTA of this row group (all experts) combines the 32 rows
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
  combine_rows<TA>(a, 0, a.T, rgo * 32, 32, tid, kK3Threads);
}

template <typename TA>
__global__ void __launch_bounds__(256) k3_combine(DownArgs<TA> a) {
  // grid: (H / 32, ceil(T / 8)); 8 tokens x 32 rows per CTA
  const int t0 = blockIdx.y * 8, t1 = min(a.T, t0 + 8);
  combine_rows<TA>(a, t0, t1, blockIdx.x * 32, 32, threadIdx.x, blockDim.x);
}

// ================================================================= launch ====
// Tokens per pass over a weight tile: an expert never has more tokens than the call.
static int tokens_per_pass(int64_t T) { return T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : 8; }

template <typename TA> int launch_combine(DownArgs<TA> &a, int64_t T, int H, cudaStream_t s);

template <typename TA, int kNT>
int launch_k3(DownArgs<TA> &a, int grid, int Kmax, cudaStream_t s) {
  const size_t smem = (size_t)kNT * Kmax * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(k3_down<TA, kNT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return cuda_check(e, "k3 smem attribute");
  }
  k3_down<TA, kNT><<<grid, kK3Threads, smem, s>>>(a);
  TM_LAUNCH_CHECK("k3_down launch");
  if (!a.combine_in_kernel) return launch_combine<TA>(a, a.T, a.H, s);
  return TM_OK;
}

template <typename TA> int launch_combine(DownArgs<TA> &a, int64_t T, int H, cudaStream_t s) {
  dim3 g(H / 32, (unsigned)((T + 7) / 8));
  k3_combine<TA><<<g, 256, 0, s>>>(a);
  TM_LAUNCH_CHECK("k3_combine launch");
  return TM_OK;
}

struct GateUpLaunch {
  const void *x; int64_t T; int H, I, E, k, Is;
  const uint8_t *w13; const float *s13; const uint8_t *sh_w13; const float *sh_s13; const void *sh_gate_w;
  void *ws; const WsLayout *L; cudaStream_t s;
  template <typename TA> int run() {
    GateUpArgs<TA> a;
    a.x = (const TA *)x;
    a.w13 = w13; a.s13 = s13; a.sh_w13 = sh_w13; a.sh_s13 = sh_s13; a.sh_gate_w = (const TA *)sh_gate_w;
    a.pl = plan_view(ws, *L);
    a.k2_cnt = ws_ptr<int>(ws, L->k2_cnt);
    a.gu_part = ws_ptr<float>(ws, L->gu_part);
    a.sh_gu_part = ws_ptr<float>(ws, L->sh_gu_part);
    a.shg_part = ws_ptr<float>(ws, L->shg_part);
    a.sh_w = ws_ptr<float>(ws, L->sh_w);
    a.h = ws_ptr<float>(ws, L->h);
    a.sh_h = ws_ptr<float>(ws, L->sh_h);
    a.T = (int)T; a.H = H; a.I = I; a.Is = sh_w13 ? Is : 0; a.E = E; a.P = (int)T * k;
    a.KQ = H / 512; a.RG = I / 32; a.RGs = a.Is / 32;
    const int max_active = (int)std::min<int64_t>(E, T * k);
    a.routed_ctas = max_active * a.RG * a.KQ;
    const int grid = a.routed_ctas + (sh_w13 ? a.RGs * a.KQ : 0);
    switch (tokens_per_pass(T)) {
      case 1: k2_gateup<TA, 1><<<grid, kK2Threads, 0, s>>>(a); break;
      case 2: k2_gateup<TA, 2><<<grid, kK2Threads, 0, s>>>(a); break;
      case 4: k2_gateup<TA, 4><<<grid, kK2Threads, 0, s>>>(a); break;
      default: k2_gateup<TA, 8><<<grid, kK2Threads, 0, s>>>(a); break;
    }
    TM_LAUNCH_CHECK("k2_gateup launch");
    return TM_OK;
  }
};

struct DownLaunch {
  int64_t T; int H, I, E, k, Is;
  const void *topk_w; const uint8_t *w2; const float *s2; const uint8_t *sh_w2; const float *sh_s2;
  const void *residual; void *out; void *ws; const WsLayout *L; cudaStream_t s;
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
    a.RGo = H / 32;
    a.has_shared = sh_w2 ? 1 : 0;
    const int max_active = (int)std::min<int64_t>(E, T * k);
    a.routed_ctas = max_active * a.RGo;
    a.combine_in_kernel = T <= kCombineInKernelMaxT ? 1 : 0;
    const int grid = a.routed_ctas + (sh_w2 ? a.RGo : 0);
    const int Kmax = std::max(I, a.Is);
    switch (tokens_per_pass(T)) {
      case 1: return launch_k3<TA, 1>(a, grid, Kmax, s);
      case 2: return launch_k3<TA, 2>(a, grid, Kmax, s);
      case 4: return launch_k3<TA, 4>(a, grid, Kmax, s);
      default: return launch_k3<TA, 8>(a, grid, Kmax, s);
    }
  }
};

}  // namespace tmoe

using namespace tmoe;

extern "C" int tm_moe_decode_gateup(const void *x, int64_t tokens, int hidden, int inter,
                                    int n_experts, int top_k, int act_dtype, const uint8_t *w13,
                                    const float *s13, const uint8_t *sh_w13, const float *sh_s13,
                                    int shared_inter, const void *sh_gate_w, void *ws,
                                    int64_t ws_bytes, void *stream) {
  TM_REQUIRE(x && w13 && s13, "null pointer");
  TM_REQUIRE(hidden % 512 == 0, "hidden (%d) must be a multiple of 512", hidden);
  TM_REQUIRE(inter % 256 == 0 && inter > 0, "inter (%d) must be a positive multiple of 256", inter);
  TM_REQUIRE(!sh_w13 || (sh_s13 && sh_gate_w && shared_inter > 0 && shared_inter % 256 == 0),
             "shared expert needs sh_s13, sh_gate_w and shared_inter %% 256 == 0");
  TM_REQUIRE(aligned(x, 16) && aligned(w13, 16) && (!sh_w13 || aligned(sh_w13, 16)),
             "x and weights must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, inter, sh_w13 ? shared_inter : 0, &L);
  if (rc) return rc;
  GateUpLaunch f{x, tokens, hidden, inter, n_experts, top_k, shared_inter, w13, s13, sh_w13, sh_s13,
                 sh_gate_w, ws, &L, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_moe_decode_down_combine(int64_t tokens, int hidden, int inter, int n_experts,
                                          int top_k, int act_dtype, const void *topk_w,
                                          const uint8_t *w2, const float *s2, const uint8_t *sh_w2,
                                          const float *sh_s2, int shared_inter, const void *residual,
                                          void *out, void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(topk_w && w2 && s2 && out, "null pointer");
  TM_REQUIRE(hidden % 512 == 0, "hidden (%d) must be a multiple of 512", hidden);
  TM_REQUIRE(inter % 256 == 0 && inter > 0, "inter (%d) must be a positive multiple of 256", inter);
  TM_REQUIRE(!sh_w2 || (sh_s2 && shared_inter > 0 && shared_inter % 256 == 0),
             "shared expert needs sh_s2 and shared_inter %% 256 == 0");
  TM_REQUIRE(aligned(w2, 16) && (!sh_w2 || aligned(sh_w2, 16)), "weights must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, inter, sh_w2 ? shared_inter : 0, &L);
  if (rc) return rc;
  DownLaunch f{tokens, hidden, inter, n_experts, top_k, shared_inter, topk_w, w2, s2, sh_w2, sh_s2,
               residual, out, ws, &L, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

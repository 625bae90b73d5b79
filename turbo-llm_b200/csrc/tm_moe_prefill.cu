// K4: prefill path (hundreds to thousands of tokens per layer call) as two
// grouped GEMMs on the 5th-generation tensor cores (tcgen05 + TMEM) and a
// combine.
//
// Reference: the multi-token branch of MoEExecutor.execute_layer
// (execution/moe.py:157-180): per active expert (ascending), gather its tokens,
// h = silu(x G^T) * (x U^T), y = h D^T, and scatter-add y * w into the output.
//
// Design (per layer call, plan from K1 in the workspace):
//   gate/up GEMM : for each (active expert, 128-row block of I, token tile)
//                  D_gate[128 x N], D_up[128 x N] = W[128 x H] . X[N x H]^T,
//                  epilogue h = silu(D_gate) * D_up -> h[slot][I] (act dtype);
//   down GEMM    : for each (active expert, 256-row block of H, token tile)
//                  D[256 x N] = W2[256 x I] . h[N x I]^T -> y[slot][H];
//   combine      : out[t] = residual[t] + sum_k w[t,k] * y[slot(t,k)].
// Weights are the MMA's A operand (M = weight rows) and tokens its N
// dimension ("swap AB"), so an expert's variable token count becomes N rounded
// up to 16 instead of padding a 128-row M tile.
//
// Weights stay FP8 in HBM and are dequantised on chip: a TMA bulk copy brings
// the raw e4m3 rows of one 64-column K slice into shared memory, eight
// converter warps turn them into bf16 (fp16) exactly as the reference's
// dequantize_weight does in that dtype (loader/expert_loader.py:150-160):
// round(cast(w) * cast(scale)).  The e4m3 byte is placed into the 16-bit
// pattern (value * 2^-120 for bf16, * 2^-8 for fp16; exact, subnormals
// included) and one bf16x2/f16x2 multiply by cast(scale) * 2^120 (2^8)
// applies the scale with a single rounding.  The tensor cores then see the
// reference's dequantised weights and the untouched activations and
// accumulate in fp32, as the reference's F.linear does.
//
// Warp roles (16 warps): 0 TMA producer, 1 TMEM owner + MMA issuer,
// 2-3 token-row gather (cp.async), 4-11 converters, 12-15 epilogue.
// Operand layouts are the UMMA K-major SWIZZLE_NONE canonical layout: 8 rows x
// 16 bytes core matrices, [k chunk][row / 8][8][16 B].  Accumulators are
// double-buffered in TMEM (2 x 256 columns) so a tile's epilogue overlaps the
// next tile's MMAs.  Every wait is bounded; on a timeout the CTA flags the
// status word, drains its copies and MMAs, frees TMEM and exits.
#include "tm_common.cuh"

namespace tmoe {

constexpr int kPfKT = 64;                        // K elements per pipeline stage
constexpr int kPfNMax = 128;                     // tokens per tile (MMA N)
constexpr int kPfRawStages = 4;
constexpr int kPfOpStages = 3;
constexpr int kPfRawBytes = 256 * kPfKT;         // 256 weight rows x 64 e4m3
constexpr int kPfABytes = 128 * kPfKT * 2;       // one 128-row 16-bit operand
constexpr int kPfBBytes = kPfNMax * kPfKT * 2;   // token rows of one stage
constexpr int kPfSmem = kPfRawStages * kPfRawBytes + kPfOpStages * (2 * kPfABytes + kPfBBytes) + 1024;
constexpr int kPfThreads = 512;
constexpr int kPfWTma = 0, kPfWMma = 1, kPfWGather = 2, kPfNGather = 2, kPfWConv = 4, kPfNConv = 8,
              kPfWEpi = 12;
constexpr int kPfTmemCols = 512;
constexpr int kPfMaxExperts = 1024;
constexpr int kPfALbo = (128 / 8) * 128;         // K-direction core-matrix stride of A

enum { kPfGateUp = 0, kPfDown = 1 };

template <typename TA> struct PfConv;
template <> struct PfConv<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;  // instruction-descriptor operand format BF16
  static constexpr int kShift = 4;     // e4m3 magnitude bits -> bf16 bits 4..10 (value * 2^-120)
  static __device__ __forceinline__ uint32_t scale(float s) {
    const float sb = __bfloat162float(__float2bfloat16_rn(s));
    const uint32_t q = __bfloat16_as_ushort(__float2bfloat16_rn(sb * 0x1p120f));
    return q | (q << 16);
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};
template <> struct PfConv<__half> {
  static constexpr uint32_t kFmt = 0;  // F16
  static constexpr int kShift = 1;     // -> f16 bits 7..13 (value * 2^-8)
  static __device__ __forceinline__ uint32_t scale(float s) {
    const float sh = __half2float(__float2half_rn(s));
    const uint32_t q = __half_as_ushort(__float2half_rn(sh * 256.f));
    return q | (q << 16);
  }
  static __device__ __forceinline__ uint32_t mul(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
  }
};

// Four e4m3 bytes -> two 16-bit pairs (bytes 0,1 -> w0; 2,3 -> w1), dequantised.
template <typename TA>
__device__ __forceinline__ void pf_convert4(uint32_t v, uint32_t S, uint32_t &w0, uint32_t &w1) {
  const uint32_t vm = v & 0x7F7F7F7Fu;
  const uint32_t a0 = __byte_perm(vm, 0, 0x1404) >> PfConv<TA>::kShift;
  const uint32_t a1 = __byte_perm(vm, 0, 0x3424) >> PfConv<TA>::kShift;
  const uint32_t s0 = __byte_perm(v, 0, 0x1404), s1 = __byte_perm(v, 0, 0x3424);
  uint32_t r0, r1;
  asm("lop3.b32 %0, %1, %2, %3, 0xD8;" : "=r"(r0) : "r"(a0), "r"(s0), "r"(0x80008000u));  // sign from s, rest a
  asm("lop3.b32 %0, %1, %2, %3, 0xD8;" : "=r"(r1) : "r"(a1), "r"(s1), "r"(0x80008000u));
  w0 = PfConv<TA>::mul(r0, S);
  w1 = PfConv<TA>::mul(r1, S);
}

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (uint64_t)((lbo >> 4) & 0x3FFF) << 16 |
         (uint64_t)((sbo >> 4) & 0x3FFF) << 32 | (uint64_t)1 << 46;  // SWIZZLE_NONE, sm100 version
}

template <typename TA> struct PfArgs {
  const TA *act;       // gate/up: x [T][H]; down: h [P][I]
  const uint8_t *w;    // packed w13 or w2 (all experts)
  const float *s;      // s13 or s2
  TA *out;             // gate/up: h [P][I]; down: y [P][H]
  const int *meta;
  const int4 *act_rec; // {expert, count, first slot, 0} per active expert
  const int *slot_token;
  uint32_t *status;
  int H, I, E;
};

struct PfTile {
  int e, slot0, nvalid, npad, mt;
};

// Tile u of the call: active experts in ascending order, then the weight-row
// block, then the token tile (fastest), so CTAs working at the same time on
// one expert's token tiles share its weight stream through L2.
__device__ __forceinline__ PfTile pf_tile(int u, const int *prefix, int na, const int4 *act_rec, int MT) {
  int lo = 0, hi = na - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= u) lo = mid;
    else hi = mid - 1;
  }
  const int4 r = __ldcg(act_rec + lo);
  const int cnt = max(r.y, 1);
  const int nt = (cnt + kPfNMax - 1) / kPfNMax;
  const int local = u - prefix[lo];
  const int mt = local / nt, j = local % nt;
  const int start = (int)((int64_t)j * cnt / nt), end = (int)((int64_t)(j + 1) * cnt / nt);
  PfTile t;
  t.e = r.x;
  t.slot0 = r.z + start;
  t.nvalid = end - start;
  t.npad = (t.nvalid + 15) & ~15;
  t.mt = mt;
  return t;
}

// Bounded wait shared by every role: false on timeout (flags the status word
// and the CTA's abort flag) or when another role has already aborted.
__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *status) {
  if (mbar_try_wait(bar, parity)) return true;
  uint64_t t0;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t0));
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63) == 0) {
      if (*abort) return false;
      uint64_t t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      if (t - t0 > 1000000000ull) {
        *abort = 1;
        atomicOr(status, TM_STATUS_TIMEOUT);
        return false;
      }
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{.reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;}" ::"r"(d),
               "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <typename TA, int kMode>
__global__ void __launch_bounds__(kPfThreads, 1) k4_gemm(PfArgs<TA> a) {
  extern __shared__ __align__(1024) uint8_t pf_smem_raw[];
  uint8_t *sm = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t *raw = sm;                                            // [kPfRawStages][kPfRawBytes]
  uint8_t *opA = raw + kPfRawStages * kPfRawBytes;              // [kPfOpStages][2][kPfABytes]
  uint8_t *opB = opA + kPfOpStages * 2 * kPfABytes;             // [kPfOpStages][kPfBBytes]
  __shared__ __align__(8) uint64_t raw_full[kPfRawStages], raw_empty[kPfRawStages];
  __shared__ __align__(8) uint64_t op_full[kPfOpStages], op_empty[kPfOpStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drain_bar;
  __shared__ int prefix[kPfMaxExperts + 1];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ int s_na, s_tiles;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool gate_up = kMode == kPfGateUp;
  const int K = gate_up ? a.H : a.I;                   // reduction length
  const int MT = gate_up ? a.I / 128 : a.H / 256;      // weight-row blocks per expert
  const int out_ld = gate_up ? a.I : a.H;
  const int nk = K / kPfKT;

  // ---- tile table: prefix[a] = first tile of active expert a ----
  if (warp == 0) {
    const int na = min(__ldcg(a.meta + kMetaNActive), a.E);
    int run = 0;
    for (int base = 0; base < na; base += 32) {
      const int i = base + lane;
      int v = 0;
      if (i < na) {
        const int cnt = max(__ldcg(&a.act_rec[i].y), 1);
        v = MT * ((cnt + kPfNMax - 1) / kPfNMax);
      }
      int incl = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      if (i < na) prefix[i] = run + incl - v;
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) {
      prefix[na] = run;
      s_na = na;
      s_tiles = run;
      abort_flag = 0;
    }
  }
  __syncthreads();
  const int na = s_na, tiles = s_tiles;
  if ((int)blockIdx.x >= tiles) return;  // CTA-uniform

  if (tid == 0) {
    for (int s = 0; s < kPfRawStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], kPfNConv * 32);
    }
    for (int s = 0; s < kPfOpStages; ++s) {
      mbar_init(&op_full[s], (kPfNConv + kPfNGather) * 32);
      mbar_init(&op_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(&drain_bar, 1);
    mbar_fence_init();
  }
  if (warp == kPfWMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(kPfTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == kPfWTma) {
    // ---------------------------------------------------- TMA producer ----
    if (lane == 0) {
      uint32_t i = 0;
      int last_parity[kPfRawStages];
      for (int s = 0; s < kPfRawStages; ++s) last_parity[s] = -1;
      for (int u = blockIdx.x; u < tiles && !abort_flag; u += gridDim.x) {
        const PfTile t = pf_tile(u, prefix, na, a.act_rec, MT);
        for (int kt = 0; kt < nk; ++kt, ++i) {
          const int rs = i % kPfRawStages;
          if (!pf_wait(&raw_empty[rs], ((i / kPfRawStages) & 1) ^ 1, &abort_flag, a.status)) break;
          mbar_arrive_expect_tx(&raw_full[rs], kPfRawBytes);
          last_parity[rs] = (i / kPfRawStages) & 1;
          uint8_t *dst = raw + rs * kPfRawBytes;
          if (gate_up) {
            // 8 row groups x (4 chunks x gate,up x 16 rows x 16 B) = 8 x 2 KB
            const uint8_t *src = a.w + (size_t)t.e * 2 * a.I * a.H + (size_t)(t.mt * 8) * 32 * a.H + (size_t)kt * 4 * 512;
            for (int g = 0; g < 8; ++g) tma_bulk_g2s(dst + g * 2048, src + (size_t)g * 32 * a.H, 2048, &raw_full[rs]);
          } else {
            // 16 row groups x (4 chunks x 16 rows x 16 B) = 16 x 1 KB
            const uint8_t *src = a.w + (size_t)t.e * a.H * a.I + (size_t)(t.mt * 16) * 16 * a.I + (size_t)kt * 4 * 256;
            for (int g = 0; g < 16; ++g) tma_bulk_g2s(dst + g * 1024, src + (size_t)g * 16 * a.I, 1024, &raw_full[rs]);
          }
        }
      }
      // drain: every armed copy must land before the CTA may exit
      volatile int no_abort = 0;
      for (int s = 0; s < kPfRawStages; ++s)
        if (last_parity[s] >= 0) pf_wait(&raw_full[s], (uint32_t)last_parity[s], &no_abort, a.status);
    }
  } else if (warp == kPfWMma) {
    // ------------------------------------------------------ MMA issuer ----
    if (lane == 0) {
      uint32_t i = 0, l = 0;
      bool issued = false;
      for (int u = blockIdx.x; u < tiles && !abort_flag; u += gridDim.x, ++l) {
        const PfTile t = pf_tile(u, prefix, na, a.act_rec, MT);
        const int b = l & 1;
        if (!pf_wait(&acc_empty[b], ((l >> 1) & 1) ^ 1, &abort_flag, a.status)) break;
        tc_fence_after();
        const uint32_t idesc = (1u << 4) | (PfConv<TA>::kFmt << 7) | (PfConv<TA>::kFmt << 10) |
                               ((uint32_t)(t.npad >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
        const uint32_t lboB = (uint32_t)(t.npad / 8) * 128;
        bool ok = true;
        for (int kt = 0; kt < nk; ++kt, ++i) {
          const int os = i % kPfOpStages;
          if (!pf_wait(&op_full[os], (i / kPfOpStages) & 1, &abort_flag, a.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t aBase = smem_u32(opA + os * 2 * kPfABytes), bBase = smem_u32(opB + os * kPfBBytes);
#pragma unroll
          for (int s = 0; s < kPfKT / 16; ++s) {
            const uint64_t bd = umma_desc(bBase + 2 * s * lboB, lboB, 128);
#pragma unroll
            for (int j = 0; j < 2; ++j) {
              const uint64_t ad = umma_desc(aBase + j * kPfABytes + 2 * s * kPfALbo, kPfALbo, 128);
              tc_mma(tmem + b * 256 + j * 128, ad, bd, idesc, (kt | s) != 0);
            }
          }
          issued = true;
          tc_commit(&op_empty[os]);
        }
        if (!ok) break;
        tc_commit(&acc_full[b]);
      }
      if (issued) {  // all MMAs of this CTA complete before TMEM may be freed
        tc_commit(&drain_bar);
        volatile int no_abort = 0;
        pf_wait(&drain_bar, 0, &no_abort, a.status);
      }
    }
  } else if (warp < kPfWConv) {
    // --------------------------------------------- token-row gather ----
    const int gt = tid - kPfWGather * 32;  // 0..63
    uint32_t i = 0;
    int prev_os = -1;
    for (int u = blockIdx.x; u < tiles && !abort_flag; u += gridDim.x) {
      const PfTile t = pf_tile(u, prefix, na, a.act_rec, MT);
      const int kc = gt & 7;
      // rows this thread copies: n = gt/8 + 8q, q < npad/8
      const TA *rows[kPfNMax / 8];
#pragma unroll
      for (int q = 0; q < kPfNMax / 8; ++q) {
        const int n = (gt >> 3) + 8 * q;
        const int slot = t.slot0 + min(n, t.nvalid - 1);
        const int r = gate_up ? __ldcg(a.slot_token + slot) : slot;
        rows[q] = a.act + (size_t)r * K + kc * 8;
      }
      bool ok = true;
      for (int kt = 0; kt < nk; ++kt, ++i) {
        const int os = i % kPfOpStages;
        if (!pf_wait(&op_empty[os], ((i / kPfOpStages) & 1) ^ 1, &abort_flag, a.status)) { ok = false; break; }
        uint8_t *dstB = opB + os * kPfBBytes;
#pragma unroll
        for (int q = 0; q < kPfNMax / 8; ++q) {
          const int n = (gt >> 3) + 8 * q;
          if (n < t.npad)
            cp_async16(dstB + (kc * (t.npad / 8) + n / 8) * 128 + (n % 8) * 16, rows[q] + kt * kPfKT);
        }
        cp_async_commit();
        if (prev_os >= 0) {
          cp_async_wait<1>();
          fence_proxy_async();
          mbar_arrive(&op_full[prev_os]);
        }
        prev_os = os;
      }
      if (!ok) break;
    }
    cp_async_wait<0>();
    if (prev_os >= 0 && !abort_flag) {
      fence_proxy_async();
      mbar_arrive(&op_full[prev_os]);
    }
  } else if (warp < kPfWEpi) {
    // ------------------------------------------------------ converters ----
    const int ct = tid - kPfWConv * 32;  // 0..255
    uint32_t i = 0;
    for (int u = blockIdx.x; u < tiles && !abort_flag; u += gridDim.x) {
      const PfTile t = pf_tile(u, prefix, na, a.act_rec, MT);
      bool ok = true;
      for (int kt = 0; kt < nk; ++kt, ++i) {
        const int rs = i % kPfRawStages, os = i % kPfOpStages;
        uint32_t S0, S1;
        if (gate_up) {
          const float *sp = a.s + ((size_t)(t.e * (a.I / 128) + t.mt) * 2) * (a.H / 128) + (kt * kPfKT) / 128;
          S0 = PfConv<TA>::scale(__ldg(sp));
          S1 = PfConv<TA>::scale(__ldg(sp + a.H / 128));
        } else {
          const float *sp = a.s + ((size_t)t.e * (a.H / 128) + t.mt * 2) * (a.I / 128) + (kt * kPfKT) / 128;
          S0 = PfConv<TA>::scale(__ldg(sp));
          S1 = PfConv<TA>::scale(__ldg(sp + a.I / 128));
        }
        if (!pf_wait(&raw_full[rs], (i / kPfRawStages) & 1, &abort_flag, a.status)) { ok = false; break; }
        if (!pf_wait(&op_empty[os], ((i / kPfOpStages) & 1) ^ 1, &abort_flag, a.status)) { ok = false; break; }
        const uint8_t *src = raw + rs * kPfRawBytes;
        uint8_t *dstA = opA + os * 2 * kPfABytes;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int p = ct + 256 * q;  // 16-byte piece of the raw stage
          int r, c, j, m;
          if (gate_up) {                // [g 8][c 4][j 2][r 16]
            r = p & 15; j = (p >> 4) & 1; c = (p >> 5) & 3; m = (p >> 7) * 16 + r;
          } else {                      // [g 16][c 4][r 16]
            r = p & 15; c = (p >> 4) & 3; const int g = p >> 6; j = g >> 3; m = (g & 7) * 16 + r;
          }
          const uint4 v = *reinterpret_cast<const uint4 *>(src + p * 16);
          const uint32_t S = j ? S1 : S0;
          uint4 lo, hi;
          pf_convert4<TA>(v.x, S, lo.x, lo.y);
          pf_convert4<TA>(v.y, S, lo.z, lo.w);
          pf_convert4<TA>(v.z, S, hi.x, hi.y);
          pf_convert4<TA>(v.w, S, hi.z, hi.w);
          uint8_t *d = dstA + j * kPfABytes + (m / 8) * 128 + (m % 8) * 16;
          *reinterpret_cast<uint4 *>(d + (2 * c) * kPfALbo) = lo;
          *reinterpret_cast<uint4 *>(d + (2 * c + 1) * kPfALbo) = hi;
        }
        mbar_arrive(&raw_empty[rs]);
        fence_proxy_async();
        mbar_arrive(&op_full[os]);
      }
      if (!ok) break;
    }
  } else {
    // -------------------------------------------------------- epilogue ----
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int m = q * 32 + lane;
    uint32_t l = 0;
    for (int u = blockIdx.x; u < tiles && !abort_flag; u += gridDim.x, ++l) {
      const PfTile t = pf_tile(u, prefix, na, a.act_rec, MT);
      const int b = l & 1;
      if (!pf_wait(&acc_full[b], (l >> 1) & 1, &abort_flag, a.status)) break;
      tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + b * 256;
      for (int c0 = 0; c0 < t.nvalid; c0 += 16) {
        float v0[16], v1[16];
        tc_ld16(tb + c0, v0);
        tc_ld16(tb + 128 + c0, v1);
        tc_wait_ld();
        if (gate_up) {
          TA *o = a.out + (size_t)(t.slot0 + c0) * out_ld + t.mt * 128 + m;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < t.nvalid) o[(size_t)j * out_ld] = Act<TA>::from_f(silu(v0[j]) * v1[j]);
        } else {
          TA *o = a.out + (size_t)(t.slot0 + c0) * out_ld + t.mt * 256 + m;
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (c0 + j < t.nvalid) {
              o[(size_t)j * out_ld] = Act<TA>::from_f(v0[j]);
              o[(size_t)j * out_ld + 128] = Act<TA>::from_f(v1[j]);
            }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[b]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kPfWMma) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kPfTmemCols));
  }
}

// out[t] = residual[t] + sum_r w[t,r] * y[slot(t,r)] (top-k order, fp32).
template <typename TA>
__global__ void __launch_bounds__(256) k4_combine(const TA *y, const TA *w, const int *pair_slot, const TA *residual,
                                                  TA *out, int H, int k) {
  const int t = blockIdx.x;
  for (int o = threadIdx.x * 8; o < H; o += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < k; ++r) {
      const int s = __ldcg(pair_slot + (size_t)t * k + r);
      if (s < 0) continue;
      const float wr = Act<TA>::to_f(w[(size_t)t * k + r]);
      const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(y + (size_t)s * H + o));
      const TA *yv = reinterpret_cast<const TA *>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = fmaf(wr, Act<TA>::to_f(yv[j]), acc[j]);
    }
    uint4 res;
    TA *rv = reinterpret_cast<TA *>(&res);
    if (residual) {
      const uint4 rr = __ldcg(reinterpret_cast<const uint4 *>(residual + (size_t)t * H + o));
      const TA *rp = reinterpret_cast<const TA *>(&rr);
#pragma unroll
      for (int j = 0; j < 8; ++j) rv[j] = Act<TA>::from_f(acc[j] + Act<TA>::to_f(rp[j]));
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) rv[j] = Act<TA>::from_f(acc[j]);
    }
    *reinterpret_cast<uint4 *>(out + (size_t)t * H + o) = res;
  }
}

static int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      n = 148;
  }
  return n;
}

struct PrefillLaunch {
  const void *x; int64_t T; int H, I, E, k;
  const void *topk_w; const uint8_t *w13; const float *s13; const uint8_t *w2; const float *s2;
  const void *residual; void *out; void *ws; const WsLayout *L; cudaStream_t s;
  template <typename TA> int run() {
    if constexpr (sizeof(TA) != 2) {
      return fail(TM_ERR_UNSUPPORTED, "tm_moe_prefill_grouped: fp32 activations are not supported (bf16, fp16)");
    } else {
      PfArgs<TA> g;
      g.meta = ws_ptr<int>(ws, L->meta);
      g.act_rec = ws_ptr<int4>(ws, L->act_rec);
      g.slot_token = ws_ptr<int>(ws, L->slot_token);
      g.status = ws_ptr<uint32_t>(ws, L->status);
      g.H = H; g.I = I; g.E = E;
      TA *h = ws_ptr<TA>(ws, L->h);        // [P][I] act dtype (region sized for fp32)
      TA *y = ws_ptr<TA>(ws, L->ypart);    // [P][H] act dtype
      const int grid = num_sms();
      g.act = (const TA *)x; g.w = w13; g.s = s13; g.out = h;
      int rc = ensure_smem(reinterpret_cast<const void *>(k4_gemm<TA, kPfGateUp>), kPfSmem);
      if (rc) return rc;
      k4_gemm<TA, kPfGateUp><<<grid, kPfThreads, kPfSmem, s>>>(g);
      TM_LAUNCH_CHECK("k4_gemm gate/up launch");
      g.act = h; g.w = w2; g.s = s2; g.out = y;
      rc = ensure_smem(reinterpret_cast<const void *>(k4_gemm<TA, kPfDown>), kPfSmem);
      if (rc) return rc;
      k4_gemm<TA, kPfDown><<<grid, kPfThreads, kPfSmem, s>>>(g);
      TM_LAUNCH_CHECK("k4_gemm down launch");
      k4_combine<TA><<<(unsigned)T, 256, 0, s>>>(y, (const TA *)topk_w, ws_ptr<int>(ws, L->pair_slot),
                                                   (const TA *)residual, (TA *)out, H, k);
      TM_LAUNCH_CHECK("k4_combine launch");
      return TM_OK;
    }
  }
};

}  // namespace tmoe

using namespace tmoe;

extern "C" int tm_moe_prefill_grouped(const void *x, int64_t tokens, int hidden, int inter, int n_experts,
                                      int top_k, int act_dtype, const void *topk_w, const uint8_t *w13,
                                      const float *s13, const uint8_t *w2, const float *s2, const void *residual,
                                      void *out, void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(x && topk_w && w13 && s13 && w2 && s2 && out, "null pointer");
  TM_REQUIRE(hidden % 256 == 0 && hidden > 0, "hidden (%d) must be a positive multiple of 256", hidden);
  TM_REQUIRE(inter % 128 == 0 && inter > 0, "inter (%d) must be a positive multiple of 128", inter);
  TM_REQUIRE(n_experts <= kPfMaxExperts, "n_experts %d > %d", n_experts, kPfMaxExperts);
  TM_REQUIRE(aligned(x, 16) && aligned(w13, 16) && aligned(w2, 16) && aligned(out, 16) &&
                 (!residual || aligned(residual, 16)),
             "x, weights, residual and out must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, inter, 0, &L);
  if (rc) return rc;
  PrefillLaunch f{x, tokens, hidden, inter, n_experts, top_k, topk_w, w13, s13, w2, s2, residual, out,
                  ws, &L, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

// K7: grouped expert GEMMs on FP8 tensor cores (tcgen05.mma kind::f8f6f4) for
// calls with few tokens per expert: expert-parallel owners (~16 rows per
// expert), batched decode of tens to hundreds of tokens, Qwen3.5-shaped calls
// with 256 experts.
//
// Reference: the multi-token branch of MoEExecutor.execute_layer
// (execution/moe.py:157-202): per active expert (ascending) its tokens'
// h = silu(x G^T) * (x U^T), y = h D^T, weighted sum in the combine, plus the
// sigmoid-gated shared expert (moe.py:191-200).
//
// Why a second grouped GEMM next to K4 (tm_moe_prefill.cu): K4 dequantises
// every weight slice into tensor memory before its MMAs, which costs the same
// whatever the token count, so with ~16 tokens per expert it runs at a third
// of the HBM bound.  Here the weights are multiplied as they are stored:
//   * A operand = raw e4m3 weights, 128 rows x 128 K bytes per tile, brought
//     into shared memory by one TMA tensor load from the packed layout of
//     tm_pack_experts (a 4-D/3-D tensor map whose box reorders the packed
//     16-row groups into the canonical no-swizzle K-major layout: 8-row core
//     matrices 128 B apart, 16-byte K chunks 2 KB apart);
//   * B operand = the tokens as two e4m3 terms, v * 2^s = hi + lo / 16 with
//     s a per-token power of 2 (bf16 values are represented exactly: 8
//     significant bits = 4 + 4, for every value within 2^-10 of the token's
//     largest); written by k7_prep in slot order, column-chunk-major
//     [K/16][rows][16 B], so each 16-byte K slab of an expert's rows is one
//     contiguous bulk copy;
//   * the fp32 block scales (one per 128 x 128 weight block) cannot enter an
//     FP8 MMA, so each 128-wide K chunk is its own MMA accumulation (D = A.B,
//     fresh per chunk, four buffers in TMEM) and the epilogue warps add
//     scale x chunk into fp32 registers: weights, scales and activations are
//     all exact, only the fp32 sums round.
// gate/up epilogue: g, u rounded to bf16, silu(g) rounded, h = silu * u
// rounded (the reference's F.linear / F.silu / * in bf16), then h of each
// (token, 128-row block) is written as two e4m3 terms with its own power of 2
// (the down GEMM's B operand and its per-chunk exponent).  down epilogue:
// y rounded to bf16 into the per-slot output rows; the combine (k4_combine)
// adds them in top-k order with the weights, the shared expert and the
// residual.
//
// Units: (active expert, 128-row weight block, group of <= 64 tokens), expert
// major, groups fastest, so CTAs working on one expert's groups at the same
// time share its weight stream through L2.  One persistent CTA per SM; warp
// 0 = TMA producer, warp 1 = TMEM owner + MMA issuer, warps 2-9 = epilogue
// (two per TMEM lane quadrant, alternate 16-column blocks).  Every wait is
// bounded (1 s); on a timeout the CTA flags TM_STATUS_TIMEOUT, drains and
// frees TMEM.  No multicast; tensor maps cover this GPU's own memory only.
#include <cuda.h>  // CUtensorMap (cuTensorMapEncodeTiled is reached through cudart)

#include <mutex>

#include "tm_common.cuh"

namespace tmoe {

constexpr int kF8GateUp = 0, kF8Down = 1;
constexpr int kF8Threads = 320;                 // 10 warps
constexpr int kF8WTma = 0, kF8WMma = 1, kF8WEpi = 2, kF8NEpi = 8;
constexpr int kF8GroupMax = 32;                 // tokens per unit (2 terms -> <= 64 MMA columns)
constexpr int kF8Tile = 128 * 128;              // one A tile (128 rows x 128 K bytes): 16 KB
constexpr int kF8BTile = 2 * kF8GroupMax * 128; // the B rows of one stage: 8 KB
constexpr int kF8ExpStride = 16;                // bytes per slot of the h exponents (I <= 2048)
constexpr int kF8MaxExperts = 1024;

template <int kMode> struct F8Cfg {
  // two A tiles per K chunk: gate and up of the same 128 rows, or two
  // 128-row halves of a 256-row block of the down projection
  static constexpr int kOps = 2;
  static constexpr int kRowsPerUnit = kMode == kF8GateUp ? 128 : 256;
  static constexpr int kStages = 5;
  static constexpr int kStageBytes = kOps * kF8Tile + kF8BTile;
  static constexpr int kSmem = kStages * kStageBytes + 1024;
  static constexpr int kAccBufs = 4;                              // accumulator buffers (MMA runs ahead)
  static constexpr int kBufCols = kOps * 2 * kF8GroupMax;         // one buffer: <= 64 columns per operand
  static constexpr int kTmemCols = kAccBufs * kBufCols;            // 512 (gate/up) or 256 (down)
};

struct F8Args {
  const uint8_t *bq;   // B rows [K/16][R][16 B]
  int64_t R;           // rows of bq (2 per slot)
  const float *s;      // routed block scales (s13 or s2)
  const float *sh_s;   // shared expert's (or NULL)
  const int *meta;
  const int4 *act_rec; // {expert, count, first slot, 0}
  const int *sexp;     // gate/up: per-slot power of 2 of the token terms
  const int8_t *hexp;  // down: per-(slot, 128-row block of I) power of 2 of the h terms, [slot][16]
  uint8_t *hq;         // gate/up output: h terms [I/16][R][16 B]
  int8_t *hexp_out;    // gate/up output: [slot][16] (entry mt of slot)
  __nv_bfloat16 *y;    // down output: [slot][H]
  uint32_t *status;
  int H, I, E, P, T, has_shared;
};

struct F8Tile {
  int e, slot0, nvalid, mt;
};

__device__ __forceinline__ F8Tile f8_tile(int u, const int *prefix, int na, int na_r, const int4 *act_rec,
                                          int4 shared_rec) {
  int lo = 0, hi = na - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= u) lo = mid;
    else hi = mid - 1;
  }
  const int4 r = lo >= na_r ? shared_rec : __ldcg(act_rec + lo);
  const int cnt = max(r.y, 1);
  const int ng = (cnt + kF8GroupMax - 1) / kF8GroupMax;
  const int local = u - prefix[lo];
  const int mt = local / ng, j = local % ng;
  const int start = (int)((int64_t)j * cnt / ng), end = (int)((int64_t)(j + 1) * cnt / ng);
  F8Tile t;
  t.e = r.x;
  t.slot0 = r.z + start;
  t.nvalid = r.y > 0 ? end - start : 0;
  t.mt = mt;
  return t;
}

__device__ __forceinline__ bool f8_wait(uint64_t *bar, uint32_t parity, volatile int *abort, uint32_t *status) {
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
__device__ __forceinline__ void f8_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void f8_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void f8_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void f8_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, e4m3 x e4m3 -> fp32
__device__ __forceinline__ void f8_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{.reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;}" ::"r"(d),
               "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
// Shared-memory descriptor, K-major, no swizzle: 8-row core matrices `sbo`
// bytes apart along M/N, the two 16-byte K halves of an MMA `lbo` bytes apart.
__device__ __forceinline__ uint64_t f8_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (uint64_t)((lbo >> 4) & 0x3FFF) << 16 |
         (uint64_t)((sbo >> 4) & 0x3FFF) << 32 | (uint64_t)1 << 46;
}
__device__ __forceinline__ void f8_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}
__device__ __forceinline__ void f8_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Tiled TMA loads (no multicast) with an L2 evict-first hint: weights stream once.
__device__ __forceinline__ void f8_tma4(void *dst, const CUtensorMap *map, int c0, int c1, int c2, int c3,
                                        uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void f8_tma3(void *dst, const CUtensorMap *map, int c0, int c1, int c2, uint64_t *bar,
                                        uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

template <int kMode>
__global__ void __launch_bounds__(kF8Threads, 1) k7_gemm(const __grid_constant__ CUtensorMap tm_w,
                                                          const __grid_constant__ CUtensorMap tm_sh, F8Args a) {
  using C = F8Cfg<kMode>;
  constexpr bool kGU = kMode == kF8GateUp;
  extern __shared__ __align__(1024) uint8_t f8_smem_raw[];
  uint8_t *stages = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(f8_smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[C::kStages], empty[C::kStages];
  __shared__ __align__(8) uint64_t acc_full[C::kAccBufs], acc_empty[C::kAccBufs], drain_bar, epi_bar;
  __shared__ int prefix[kF8MaxExperts + 2];
  __shared__ float red[4][kF8GroupMax];  // gate/up: per-quadrant max |h| of each token of the unit
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ int s_na, s_na_r, s_units;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int M = kGU ? a.I : a.H;     // weight rows per expert
  const int K = kGU ? a.H : a.I;     // reduction length
  const int MB = M / 128;            // 128-row blocks (of the block scales)
  const int MT = M / C::kRowsPerUnit, KC = K / 128;
  const int4 shared_rec = make_int4(a.E, a.T, a.P, 0);

  if (warp == 0) {
    const int na_r = min(__ldcg(a.meta + kMetaNActive), a.E);
    const int na = na_r + (a.has_shared ? 1 : 0);
    int run = 0;
    for (int base = 0; base < na; base += 32) {
      const int i = base + lane;
      int v = 0;
      if (i < na) {
        const int cnt = max(i >= na_r ? a.T : __ldcg(&a.act_rec[i].y), 1);
        v = MT * ((cnt + kF8GroupMax - 1) / kF8GroupMax);
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
      s_na_r = na_r;
      s_units = run;
      abort_flag = 0;
    }
  }
  __syncthreads();
  const int na = s_na, na_r = s_na_r, units = s_units;
  if ((int)blockIdx.x >= units) return;  // CTA-uniform
  const int n_local = (units - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  auto tile_at = [&](int j) { return f8_tile(blockIdx.x + j * gridDim.x, prefix, na, na_r, a.act_rec, shared_rec); };

  if (tid == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < C::kAccBufs; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kF8NEpi);
    }
    mbar_init(&drain_bar, 1);
    mbar_init(&epi_bar, kF8NEpi);
    mbar_fence_init();
  }
  if (warp == kF8WMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  f8_fence_before();
  __syncthreads();
  f8_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == kF8WTma) {
    // ------------------------------------------------------ TMA producer ----
    // lane 0 waits for the stage and issues the weight tiles; lanes 0-7 each
    // copy one 16-byte K slab of the unit's token rows
    const uint64_t pol = l2_evict_first();
    uint32_t it = 0;
    bool ok = true;
    for (int j = 0; j < n_local && ok; ++j) {
      const F8Tile t = tile_at(j);
      const bool sh = t.e == a.E;
      const CUtensorMap *map = sh ? &tm_sh : &tm_w;
      const int g0 = (sh ? 0 : t.e * (M / 16)) + t.mt * (C::kRowsPerUnit / 16);   // first 16-row group
      const uint32_t slab = (uint32_t)t.nvalid * 2 * 16;      // bytes of one 16-byte K slab of the rows
      const uint32_t ncol = (uint32_t)((t.nvalid * 2 + 15) & ~15);
      const uint8_t *bsrc = a.bq + (size_t)t.slot0 * 2 * 16;
      for (int kc = 0; kc < KC; ++kc, ++it) {
        const int st = it % C::kStages;
        bool got = true;
        if (lane == 0) got = f8_wait(&empty[st], ((it / C::kStages) & 1) ^ 1, &abort_flag, a.status);
        if (!__shfl_sync(0xffffffffu, (int)got, 0)) { ok = false; break; }
        uint8_t *sbase = stages + st * C::kStageBytes;
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[st], (uint32_t)(C::kOps * kF8Tile) + 8 * slab);
          if constexpr (kGU) {
            f8_tma4(sbase, map, 0, g0, kc * 8, 0, &full[st], pol);
            f8_tma4(sbase + kF8Tile, map, 0, g0, kc * 8, 1, &full[st], pol);
          } else {
            f8_tma3(sbase, map, 0, g0, kc * 8, &full[st], pol);
            f8_tma3(sbase + kF8Tile, map, 0, g0 + 8, kc * 8, &full[st], pol);
          }
        }
        __syncwarp();   // the expected byte count is set before any slab copy can complete
        if (slab && lane < 8)
          tma_bulk_g2s(sbase + C::kOps * kF8Tile + lane * ncol * 16, bsrc + (size_t)(kc * 8 + lane) * a.R * 16, slab,
                       &full[st]);
      }
    }
    // no copy may still be landing in shared memory when the CTA exits
    // (after an abort the MMA warp stops consuming stages)
    if (lane == 0)
      for (uint32_t i = it > (uint32_t)C::kStages ? it - C::kStages : 0; i < it; ++i) {
        volatile int no_abort = 0;
        f8_wait(&full[i % C::kStages], (i / C::kStages) & 1, &no_abort, a.status);
      }
  } else if (warp == kF8WMma) {
    // ------------------------------------------------------- MMA issuer ----
    if (lane == 0) {
      uint32_t it = 0, ch = 0;
      bool ok = true, issued = false;
      for (int j = 0; j < n_local && ok; ++j) {
        const F8Tile t = tile_at(j);
        const uint32_t ncol = (uint32_t)((t.nvalid * 2 + 15) & ~15);
        const uint32_t n_mma = ncol < 16 ? 16 : ncol;
        const uint32_t idesc = (1u << 4) | ((n_mma >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
        for (int kc = 0; kc < KC; ++kc, ++it, ++ch) {
          const int buf = ch % C::kAccBufs, st = it % C::kStages;
          if (!f8_wait(&acc_empty[buf], ((ch / C::kAccBufs) & 1) ^ 1, &abort_flag, a.status) ||
              !f8_wait(&full[st], (it / C::kStages) & 1, &abort_flag, a.status)) { ok = false; break; }
          f8_fence_after();
          const uint32_t sbase = smem_u32(stages + st * C::kStageBytes);
          const uint32_t bbase = sbase + C::kOps * kF8Tile;
#pragma unroll
          for (int s = 0; s < 4; ++s) {
            const uint64_t bd = f8_desc(bbase + (uint32_t)(2 * s) * n_mma * 16, n_mma * 16, 128);
#pragma unroll
            for (int op = 0; op < C::kOps; ++op) {
              const uint64_t ad = f8_desc(sbase + op * kF8Tile + (uint32_t)(2 * s) * 2048, 2048, 128);
              f8_mma(tmem + buf * C::kBufCols + op * (2 * kF8GroupMax), ad, bd, idesc, s > 0);
            }
          }
          issued = true;
          f8_commit(&empty[st]);
          f8_commit(&acc_full[buf]);
        }
      }
      if (issued) {  // every MMA of this CTA completes before TMEM may be freed
        f8_commit(&drain_bar);
        volatile int no_abort = 0;
        f8_wait(&drain_bar, 0, &no_abort, a.status);
      }
    }
  } else {
    // --------------------------------------------------------- epilogue ----
    const int q = warp & 3;                    // TMEM lane quadrant
    const int hf = (warp - kF8WEpi) >> 2;      // 16-column block hf (tokens 8 hf .. 8 hf + 7) and hf + 2
    const int m = q * 32 + lane;               // weight row within the block
    const uint32_t tq = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t ch = 0, ep = 0;  // accumulator chunks consumed, epilogue-barrier phases passed
    // the 8 epilogue warps meet (bounded: a warp that aborted makes the others time out, never hang)
    auto epi_sync = [&]() -> bool {
      __syncwarp();
      if (lane == 0) f8_arrive(&epi_bar);
      const bool r = f8_wait(&epi_bar, ep & 1, &abort_flag, a.status);
      ++ep;
      return r;
    };
    for (int j = 0; j < n_local && !abort_flag; ++j) {
      const F8Tile t = tile_at(j);
      const bool sh = t.e == a.E;
      const int nblk = (t.nvalid * 2 + 15) >> 4;
      float acc[C::kOps][2][16];
#pragma unroll
      for (int op = 0; op < C::kOps; ++op)
#pragma unroll
        for (int bi = 0; bi < 2; ++bi)
#pragma unroll
          for (int c = 0; c < 16; ++c) acc[op][bi][c] = 0.f;
      // block scales of this unit, lane l holding chunks l, l + 32, ...:
      // gate/up s13 [E][I/128][2][H/128]; down s2 [E][H/128][I/128]
      const float *sc = kGU ? (sh ? a.sh_s : a.s + (size_t)t.e * MB * 2 * KC) + (size_t)t.mt * 2 * KC
                            : (sh ? a.sh_s : a.s + (size_t)t.e * MB * KC) + (size_t)t.mt * 2 * KC;
      float scr[C::kOps][4];
#pragma unroll
      for (int op = 0; op < C::kOps; ++op)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int kc = lane + 32 * u;
          scr[op][u] = kc < KC ? __ldg(sc + op * KC + kc) : 0.f;
        }
      // down: h exponents of the tokens of this lane's columns (lanes 0-15: column l of each block)
      uint4 hx[2] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};
      if constexpr (!kGU) {
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int tok = (hf + 2 * bi) * 8 + (lane >> 1);
          if (lane < 16 && tok < t.nvalid)
            hx[bi] = __ldcg(reinterpret_cast<const uint4 *>(a.hexp + (size_t)(t.slot0 + tok) * kF8ExpStride));
        }
      }
      bool ok = true;
      for (int kc = 0; kc < KC; ++kc, ++ch) {
        const int buf = ch % C::kAccBufs;
        if (!__all_sync(0xffffffffu, f8_wait(&acc_full[buf], (ch / C::kAccBufs) & 1, &abort_flag, a.status))) {
          ok = false;
          break;
        }
        f8_fence_after();
        float s_op[C::kOps];
#pragma unroll
        for (int op = 0; op < C::kOps; ++op) {
          float sv = scr[op][0];
#pragma unroll
          for (int u = 1; u < 4; ++u)
            if ((kc >> 5) == u) sv = scr[op][u];
          s_op[op] = __shfl_sync(0xffffffffu, sv, kc & 31);
        }
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int b = hf + 2 * bi;
          if (b < nblk) {
            float v[C::kOps][16];
#pragma unroll
            for (int op = 0; op < C::kOps; ++op)
              f8_ld16(tq + buf * C::kBufCols + op * (2 * kF8GroupMax) + b * 16, v[op]);
            f8_wait_ld();
            float colf = 1.f;   // down: this lane's column power of 2 of the h terms of chunk kc
            if constexpr (!kGU) {
              const uint32_t wd = kc < 4 ? hx[bi].x : kc < 8 ? hx[bi].y : kc < 12 ? hx[bi].z : hx[bi].w;
              colf = ldexpf(1.f, -(int)(int8_t)((wd >> (8 * (kc & 3))) & 0xFFu));
            }
#pragma unroll
            for (int op = 0; op < C::kOps; ++op)
#pragma unroll
              for (int c = 0; c < 16; ++c) {
                const float f = kGU ? s_op[op] : s_op[op] * __shfl_sync(0xffffffffu, colf, c);
                acc[op][bi][c] = fmaf(v[op][c], f, acc[op][bi][c]);
              }
          }
        }
        f8_fence_before();
        __syncwarp();
        if (lane == 0) f8_arrive(&acc_empty[buf]);
      }
      if (!ok) break;
      // ---- finish the unit ----
      if constexpr (kGU) {
        // h per (row m, token), the reference's bf16 roundings; lane l < nvalid
        // holds token l's power of 2 of the x terms
        const int my_sx = lane < t.nvalid ? __ldcg(a.sexp + t.slot0 + lane) : 0;
        float hv[2][8];
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int b = hf + 2 * bi;
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int tok = b * 8 + p;
            const int sx = __shfl_sync(0xffffffffu, my_sx, tok & 31);
            float h = 0.f;
            if (b < nblk && tok < t.nvalid) {
              const float f = ldexpf(1.f, -sx);
              const float g = Act<__nv_bfloat16>::round((acc[0][bi][2 * p] + acc[0][bi][2 * p + 1] * 0.0625f) * f);
              const float u = Act<__nv_bfloat16>::round((acc[1][bi][2 * p] + acc[1][bi][2 * p + 1] * 0.0625f) * f);
              const float sg = Act<__nv_bfloat16>::round(g / (1.0f + expf(-g)));
              h = Act<__nv_bfloat16>::round(sg * u);
            }
            hv[bi][p] = h;
            float mx = fabsf(h);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            if (lane == 0 && b < nblk) red[q][tok] = mx;
          }
        }
        if (!__all_sync(0xffffffffu, epi_sync())) break;
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int b = hf + 2 * bi;
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int tok = b * 8 + p;
            if (b < nblk && tok < t.nvalid) {
              const float mx = fmaxf(fmaxf(red[0][tok], red[1][tok]), fmaxf(red[2][tok], red[3][tok]));
              const int e = e4m3_shift(mx);
              const float v = ldexpf(hv[bi][p], e);
              const uint32_t hi = e4m3x2_from(v, 0.f) & 0xFFu;
              const float r = (v - e4m3x2_value(hi).x) * 16.f;
              const uint32_t lo = e4m3x2_from(r, 0.f) & 0xFFu;
              const int slot = t.slot0 + tok;
              uint8_t *dst = a.hq + ((size_t)(t.mt * 8 + (m >> 4)) * a.R + (size_t)slot * 2) * 16 + (m & 15);
              dst[0] = (uint8_t)hi;
              dst[16] = (uint8_t)lo;
              if (m == 0) a.hexp_out[(size_t)slot * kF8ExpStride + t.mt] = (int8_t)e;
            }
          }
        }
        if (!__all_sync(0xffffffffu, epi_sync())) break;  // red[] is reused by the next unit
      } else {
#pragma unroll
        for (int bi = 0; bi < 2; ++bi) {
          const int b = hf + 2 * bi;
#pragma unroll
          for (int p = 0; p < 8; ++p) {
            const int tok = b * 8 + p;
            if (b < nblk && tok < t.nvalid) {
#pragma unroll
              for (int op = 0; op < C::kOps; ++op) {
                const float y = acc[op][bi][2 * p] + acc[op][bi][2 * p + 1] * 0.0625f;
                a.y[(size_t)(t.slot0 + tok) * a.H + t.mt * 256 + op * 128 + m] = __float2bfloat16_rn(y);
              }
            }
          }
        }
      }
    }
  }

  f8_fence_before();
  __syncthreads();
  if (warp == kF8WMma) {
    f8_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
}

// ------------------------------------------------------------------ prep ----
// One warp per B row pair (slot): the slot's token row x -> s = power of 2
// putting max |x| in [128, 256), v = x * 2^s split into hi + lo / 16 (two
// e4m3 terms, exact for bf16 values), rows 2 * slot and 2 * slot + 1 of bq
// [H/16][R][16 B]; sexp[slot] = s.  Shared-expert slots [P, P + T) hold token
// slot - P and also compute its gate score sh_w[t] = sigmoid(x . g) (the
// F.linear output and the sigmoid rounded to bf16, moe.py:196-198).
__global__ void __launch_bounds__(256) k7_prep(const __nv_bfloat16 *x, const int *slot_token, const int *meta,
                                               int P, int T, int H, int has_shared, const __nv_bfloat16 *sh_gate_w,
                                               float *sh_w, uint8_t *bq, int64_t R, int *sexp) {
  const int lane = threadIdx.x & 31;
  const int slot = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int Rt = P + (has_shared ? T : 0);
  if (slot >= Rt) return;
  if (slot < P && slot >= __ldcg(meta + kMetaPairs)) return;  // no routed pair in this slot
  const int t = slot < P ? __ldcg(slot_token + slot) : slot - P;
  const uint4 *xr = reinterpret_cast<const uint4 *>(x + (size_t)t * H);
  const bool gate = slot >= P && sh_gate_w != nullptr;
  const uint4 *gr = reinterpret_cast<const uint4 *>(sh_gate_w);
  const int nv = H / 8;
  float mx = 0.f, gl = 0.f;
  for (int i = lane; i < nv; i += 32) {
    const uint4 v = __ldcg(xr + i);
    const __nv_bfloat16 *p = reinterpret_cast<const __nv_bfloat16 *>(&v);
    if (gate) {
      const uint4 gv = __ldg(gr + i);
      const __nv_bfloat16 *gp = reinterpret_cast<const __nv_bfloat16 *>(&gv);
#pragma unroll
      for (int j = 0; j < 8; ++j) gl = fmaf(__bfloat162float(p[j]), __bfloat162float(gp[j]), gl);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(__bfloat162float(p[j])));
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    gl += __shfl_xor_sync(0xffffffffu, gl, o);
  }
  if (gate && lane == 0) {
    const float logit = Act<__nv_bfloat16>::round(gl);
    sh_w[t] = Act<__nv_bfloat16>::round(1.0f / (1.0f + __expf(-logit)));
  }
  const int s = e4m3_shift(mx);
  if (lane == 0) sexp[slot] = s;
  // 16-element K slabs: lane takes slabs lane, lane + 32, ...
  for (int kk = lane; kk < H / 16; kk += 32) {
    const uint4 v0 = __ldcg(xr + 2 * kk), v1 = __ldcg(xr + 2 * kk + 1);
    const __nv_bfloat16 *p0 = reinterpret_cast<const __nv_bfloat16 *>(&v0);
    const __nv_bfloat16 *p1 = reinterpret_cast<const __nv_bfloat16 *>(&v1);
    float v[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = ldexpf(__bfloat162float(p0[j]), s);
      v[8 + j] = ldexpf(__bfloat162float(p1[j]), s);
    }
    uint32_t hi[4], lo[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      hi[w] = e4m3x2_from(v[4 * w], v[4 * w + 1]) | (e4m3x2_from(v[4 * w + 2], v[4 * w + 3]) << 16);
      const float2 a = e4m3x2_value(hi[w] & 0xFFFFu), b = e4m3x2_value(hi[w] >> 16);
      lo[w] = e4m3x2_from((v[4 * w] - a.x) * 16.f, (v[4 * w + 1] - a.y) * 16.f) |
              (e4m3x2_from((v[4 * w + 2] - b.x) * 16.f, (v[4 * w + 3] - b.y) * 16.f) << 16);
    }
    uint4 *dst = reinterpret_cast<uint4 *>(bq + ((size_t)kk * R + (size_t)slot * 2) * 16);
    dst[0] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    dst[1] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
  }
}

// ---------------------------------------------------------- tensor maps ----
using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static int encode_fn(EncodeTiledFn *out) {
  static EncodeTiledFn fn = nullptr;
  static std::mutex mu;
  std::lock_guard<std::mutex> g(mu);
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
    int rc = cuda_check(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q),
                        "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (rc) return rc;
    if (!p || q != cudaDriverEntryPointSuccess) return fail(TM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  *out = fn;
  return TM_OK;
}

// Packed gate/up weights of `experts` experts as (256 B of a 16-row group,
// row group, 16-byte K chunk, gate/up) -> box (256, 8, 8, 1) = one 128 x 128
// tile in the canonical layout; packed down weights as (256 B, row group,
// K chunk) -> box (256, 8, 8).
static int weight_map(CUtensorMap *m, const uint8_t *w, int experts, int rows, int K, bool gate_up) {
  EncodeTiledFn fn;
  int rc = encode_fn(&fn);
  if (rc) return rc;
  const cuuint64_t groups = (cuuint64_t)experts * (rows / 16), chunks = (cuuint64_t)(K / 16);
  CUresult r;
  if (gate_up) {
    const cuuint64_t dims[4] = {256, groups, chunks, 2};
    const cuuint64_t strides[3] = {chunks * 512, 512, 256};
    const cuuint32_t box[4] = {256, 8, 8, 1};
    const cuuint32_t es[4] = {1, 1, 1, 1};
    r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<uint8_t *>(w), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    const cuuint64_t dims[3] = {256, groups, chunks};
    const cuuint64_t strides[2] = {chunks * 256, 256};
    const cuuint32_t box[3] = {256, 8, 8};
    const cuuint32_t es[3] = {1, 1, 1};
    r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(w), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) return fail(TM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TM_OK;
}

static int f8_num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      n = 148;
  }
  return n;
}

// Per-slot expert outputs (bf16, slot order) of the plan in `ws`, left in the
// ypart region as [Rt][H]; Rt = P (+ T with a shared expert).  Workspace use:
// ypart = y [Rt][H] bf16, then the token terms [H/16][2 Rt][16 B]; h region =
// h terms [I/16][2 Rt][16 B], then their exponents [Rt][16]; logits region
// = per-slot token exponents [Rt]; sh_w = shared gate scores [T].
int f8_expert_outputs(const void *x, int64_t T, int H, int I, int E, int k, const uint8_t *w13, const float *s13,
                      const uint8_t *w2, const float *s2, const uint8_t *sh_w13, const float *sh_s13,
                      const uint8_t *sh_w2, const float *sh_s2, const void *sh_gate_w, void *ws, const WsLayout &L,
                      cudaStream_t s) {
  TM_REQUIRE(H % 256 == 0 && I % 128 == 0 && H >= 256 && I >= 128, "hidden %d (multiple of 256) / inter %d "
             "(multiple of 128) unsupported", H, I);
  TM_REQUIRE(E <= kF8MaxExperts, "n_experts %d > %d", E, kF8MaxExperts);
  const bool shared = sh_w13 != nullptr;
  const int64_t P = T * k, Rt = P + (shared ? T : 0), R = 2 * Rt;
  TM_REQUIRE(Rt < (1 << 30) && R * (int64_t)(H / 16) < ((int64_t)1 << 40), "call too large");
  // the regions (sized for K4's fp32 buffers) hold these
  TM_REQUIRE(I <= 128 * kF8ExpStride, "inter %d > %d", I, 128 * kF8ExpStride);
  TM_REQUIRE(Rt * H * 2 + R * H <= L.total - L.ypart && R * I + Rt * kF8ExpStride <= L.ypart - L.h &&
                 Rt * 4 <= L.counts - L.logits,
             "workspace regions too small for the FP8 grouped GEMMs");
  __nv_bfloat16 *y = ws_ptr<__nv_bfloat16>(ws, L.ypart);
  uint8_t *xq = reinterpret_cast<uint8_t *>(y) + (size_t)Rt * H * 2;
  uint8_t *hq = ws_ptr<uint8_t>(ws, L.h);
  int8_t *hexp = reinterpret_cast<int8_t *>(hq + (size_t)R * I);   // [Rt][16]
  int *sexp = ws_ptr<int>(ws, L.logits);
  float *sh_w = ws_ptr<float>(ws, L.sh_w);
  k7_prep<<<(unsigned)((Rt + 7) / 8), 256, 0, s>>>((const __nv_bfloat16 *)x, ws_ptr<int>(ws, L.slot_token),
                                                    ws_ptr<int>(ws, L.meta), (int)P, (int)T, H, shared ? 1 : 0,
                                                    (const __nv_bfloat16 *)sh_gate_w, sh_w, xq, R, sexp);
  TM_LAUNCH_CHECK("k7_prep launch");
  CUtensorMap m_gu, m_gu_sh, m_d, m_d_sh;
  int rc = weight_map(&m_gu, w13, E, I, H, true);
  if (!rc) rc = weight_map(&m_gu_sh, shared ? sh_w13 : w13, 1, I, H, true);
  if (!rc) rc = weight_map(&m_d, w2, E, H, I, false);
  if (!rc) rc = weight_map(&m_d_sh, shared ? sh_w2 : w2, 1, H, I, false);
  if (rc) return rc;
  F8Args g;
  g.R = R;
  g.meta = ws_ptr<int>(ws, L.meta);
  g.act_rec = ws_ptr<int4>(ws, L.act_rec);
  g.sexp = sexp;
  g.hexp = hexp;
  g.hq = hq;
  g.hexp_out = hexp;
  g.y = y;
  g.status = ws_ptr<uint32_t>(ws, L.status);
  g.H = H; g.I = I; g.E = E; g.P = (int)P; g.T = (int)T; g.has_shared = shared ? 1 : 0;
  const int grid = f8_num_sms();
  g.bq = xq; g.s = s13; g.sh_s = shared ? sh_s13 : nullptr;
  rc = ensure_smem(reinterpret_cast<const void *>(k7_gemm<kF8GateUp>), F8Cfg<kF8GateUp>::kSmem);
  if (rc) return rc;
  k7_gemm<kF8GateUp><<<grid, kF8Threads, F8Cfg<kF8GateUp>::kSmem, s>>>(m_gu, m_gu_sh, g);
  TM_LAUNCH_CHECK("k7_gemm gate/up launch");
  g.bq = hq; g.s = s2; g.sh_s = shared ? sh_s2 : nullptr;
  rc = ensure_smem(reinterpret_cast<const void *>(k7_gemm<kF8Down>), F8Cfg<kF8Down>::kSmem);
  if (rc) return rc;
  k7_gemm<kF8Down><<<grid, kF8Threads, F8Cfg<kF8Down>::kSmem, s>>>(m_d, m_d_sh, g);
  TM_LAUNCH_CHECK("k7_gemm down launch");
  return TM_OK;
}

}  // namespace tmoe

using namespace tmoe;

extern "C" int tm_moe_grouped_f8(const void *x, int64_t tokens, int hidden, int inter, int n_experts, int top_k,
                                 int act_dtype, const void *topk_w, const uint8_t *w13, const float *s13,
                                 const uint8_t *w2, const float *s2, const uint8_t *sh_w13, const float *sh_s13,
                                 const uint8_t *sh_w2, const float *sh_s2, int shared_inter, const void *sh_gate_w,
                                 const void *residual, void *out, void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(x && topk_w && w13 && s13 && w2 && s2 && out, "null pointer");
  TM_REQUIRE(act_dtype == TM_DTYPE_BF16, "tm_moe_grouped_f8: bf16 activations only (fp16: tm_moe_prefill_grouped)");
  const bool shared = sh_w13 != nullptr;
  TM_REQUIRE(!shared || (sh_s13 && sh_w2 && sh_s2 && sh_gate_w), "shared expert: every pointer or none");
  if (shared) {
    TM_REQUIRE(shared_inter == inter, "shared expert inter %d != inter %d", shared_inter, inter);
    TM_REQUIRE(n_experts > top_k, "shared expert needs n_experts > top_k");
    TM_REQUIRE(aligned(sh_w13, 16) && aligned(sh_w2, 16) && aligned(sh_gate_w, 16),
               "shared weights must be 16-byte aligned");
  }
  TM_REQUIRE(hidden % 256 == 0 && hidden >= 256 && inter % 128 == 0 && inter >= 128,
             "hidden (%d) must be a multiple of 256 and inter (%d) of 128", hidden, inter);
  TM_REQUIRE(top_k >= 1 && top_k <= 64, "top_k %d outside [1, 64]", top_k);
  TM_REQUIRE(aligned(x, 16) && aligned(w13, 16) && aligned(w2, 16) && aligned(out, 16) &&
                 (!residual || aligned(residual, 16)),
             "x, weights, residual and out must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, inter, shared ? shared_inter : 0, &L);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  rc = f8_expert_outputs(x, tokens, hidden, inter, n_experts, top_k, w13, s13, w2, s2, sh_w13, sh_s13, sh_w2, sh_s2,
                         sh_gate_w, ws, L, s);
  if (rc) return rc;
  const int64_t P = tokens * top_k;
  return combine_expert_outputs(ws_ptr<void>(ws, L.ypart), topk_w, ws_ptr<int>(ws, L.pair_slot), residual, out,
                                tokens, hidden, top_k, act_dtype, shared ? ws_ptr<float>(ws, L.sh_w) : nullptr,
                                (int)P, s);
}

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
// Where the bytes go.  A tcgen05.mma with both operands in shared memory is
// limited by shared-memory bandwidth (128 B/cycle/SM) whenever N < 256: it
// reads (128 + N) x 32 bytes per K=16 step.  So operand A, the dequantised
// weights, never passes through shared memory: a producer warp copies the raw
// e4m3 rows of each 64-column K slice into a ring of shared-memory stages by
// TMA bulk copies (several slices in flight, 1 byte per weight), eight
// converter warps dequantise them in registers and write them to tensor
// memory with tcgen05.st; the MMA reads A from TMEM and only the token rows
// (B) from shared memory.
//
// Dequantisation.  f16 operands (gate/up always; down for fp16 activations):
// the hardware e4m3x2 -> f16x2 conversion (exact) and one f16x2 multiply by
// f16(scale * 2^kw).  For fp16 activations kw = 0 and this is the reference's
// fp16 dequantize_weight (loader/expert_loader.py:150-160) bit for bit; for
// bf16 activations the gate/up GEMM runs on f16 (activations shifted by an
// exact per-token power of 2, weights by 2^8; both undone in the epilogue).
// bf16 down projection: bf16 weights exactly as the reference's bf16
// dequantisation, round(cast(w) * cast(scale)) (pf_convert4_bf16).  The tensor
// cores accumulate in fp32, as the reference's F.linear does.
//
// Warp roles (20 warps): 0 raw weight slices by TMA, 1 TMEM owner + MMA
// issuer, 2-3 token-row gather (cp.async into the K-major 128-byte-swizzle
// layout, several stages in flight), 4-11 converters (warp w: operand
// (w - 4) / 4, TMEM lane quadrant w % 4), 12-19 epilogue (two warps per lane
// quadrant, alternate 16-column chunks).  TMEM: columns
// [0, 128) hold the A ring (2 stages x 2 operands x 32 columns), [128, 512)
// the accumulators: tiles of <= 96 tokens alternate between two 192-column
// slots (the epilogue of one overlaps the MMAs of the next), larger tiles
// (<= 192 tokens) use both.  Every wait is bounded; on a timeout the CTA
// flags the status word, drains its copies and MMAs, frees TMEM and exits.
#include "tm_common.cuh"

namespace tmoe {

constexpr int kPfKT = 64;                        // K elements per pipeline stage
constexpr int kPfNMax = 192;                     // tokens per tile (MMA N; <= 2 x kPfNSmall)
constexpr int kPfNSmall = 96;                    // tiles up to this size double-buffer their accumulators
constexpr int kPfAStages = 2;                    // dequantised weight slices in TMEM (converters -> MMA)
constexpr int kPfBStages = 5;                    // token-row slices in shared memory (gather -> MMA)
constexpr int kPfGatherLag = 3;                  // gather stages in flight (< kPfBStages)
constexpr int kPfWStages = 6;                    // raw e4m3 weight slices in shared memory (TMA -> converters)
constexpr int kPfWBytes = 16384;                 // one raw slice: 128 rows x 64 bytes x 2 operands, or 256 x 64
constexpr int kPfBBytes = kPfNMax * kPfKT * 2;   // token rows of one stage (24 KB)
constexpr int kPfSmem = kPfBStages * kPfBBytes + kPfWStages * kPfWBytes + 1024;
constexpr int kPfWPre = 0, kPfWMma = 1, kPfWGather = 2, kPfNGather = 2, kPfWConv = 4, kPfNConv = 8,
              kPfWEpi = 12, kPfNEpi = 8;
constexpr int kPfThreads = (kPfWEpi + kPfNEpi) * 32;
constexpr int kPfTmemCols = 512;
constexpr int kPfAccBase = kPfAStages * 64;      // first accumulator column
constexpr int kPfSlotCols = 2 * kPfNSmall;       // one accumulator slot (gate + up of <= 96 tokens)
static_assert(kPfAccBase + 2 * kPfSlotCols <= kPfTmemCols, "A ring + two accumulator slots fit in TMEM");
constexpr int kPfMaxExperts = 1024;
constexpr int kPfMaxKBlocks = 128;               // K <= 16384
constexpr int kPfMaxLocalTiles = 32;             // tile descriptors cached in shared memory

enum { kPfGateUp = 0, kPfDown = 1 };

template <typename TA> struct PfConv;
template <> struct PfConv<__nv_bfloat16> {
  static constexpr uint32_t kFmt = 1;  // instruction-descriptor operand format BF16
  static __device__ __forceinline__ uint32_t scale(float s) {  // bf16(s) * 2^112, exact
    const float sb = __bfloat162float(__float2bfloat16_rn(s));
    const uint32_t q = __bfloat16_as_ushort(__float2bfloat16_rn(sb * 0x1p112f));
    return q | (q << 16);
  }
};
template <> struct PfConv<__half> {
  static constexpr uint32_t kFmt = 0;  // F16
};

// f16 weights: round_f16(w * f16(scale * 2^kw)).
__device__ __forceinline__ uint32_t pf_scale_f16(float s, int kw) {
  const uint32_t q = __half_as_ushort(__float2half_rn(ldexpf(s, kw)));
  return q | (q << 16);
}
__device__ __forceinline__ void pf_convert4_f16(uint32_t v, uint32_t S, uint32_t &w0, uint32_t &w1) {
  uint32_t h0, h1;
  asm("{\n\t.reg .b16 p, q;\n\tmov.b32 {p, q}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, p;\n\tcvt.rn.f16x2.e4m3x2 %1, q;\n\t}"
      : "=r"(h0), "=r"(h1)
      : "r"(v));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(w0) : "r"(h0), "r"(S));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(w1) : "r"(h1), "r"(S));
}
// bf16 weights (reference-exact): bytes 0,1 -> w0; 2,3 -> w1.  The exact f16
// image of each e4m3 value has its 7 low mantissa bits zero, so shifting the
// f16 magnitude right by 3 yields a bf16 pattern of value * 2^-112 (exponent
// rebiased by the bf16 - f16 bias difference, never subnormal); the sign is
// merged back and one bf16x2 multiply by bf16(scale) * 2^112 applies the
// scale with a single rounding.  (Only an e4m3 NaN byte, absent from finite
// checkpoints, would disturb its pair neighbour.)
__device__ __forceinline__ void pf_convert4_bf16(uint32_t v, uint32_t S, uint32_t &w0, uint32_t &w1) {
  uint32_t h0, h1;
  asm("{\n\t.reg .b16 p, q;\n\tmov.b32 {p, q}, %2;\n\t"
      "cvt.rn.f16x2.e4m3x2 %0, p;\n\tcvt.rn.f16x2.e4m3x2 %1, q;\n\t}"
      : "=r"(h0), "=r"(h1)
      : "r"(v));
  uint32_t r0, r1;
  asm("lop3.b32 %0, %1, %2, %3, 0xD8;" : "=r"(r0) : "r"((h0 & 0x7FFF7FFFu) >> 3), "r"(h0), "r"(0x80008000u));
  asm("lop3.b32 %0, %1, %2, %3, 0xD8;" : "=r"(r1) : "r"((h1 & 0x7FFF7FFFu) >> 3), "r"(h1), "r"(0x80008000u));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(w0) : "r"(r0), "r"(S));
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(w1) : "r"(r1), "r"(S));
}

// UMMA shared-memory descriptor, K-major 128-byte swizzle: 8-row groups 1024 B
// apart (SBO), LBO unused (16 B), sm100 version bit 46.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFF) | (uint64_t)1 << 16 | (uint64_t)(1024 >> 4) << 32 | (uint64_t)1 << 46 |
         (uint64_t)2 << 61;
}

template <typename TA> struct PfArgs {
  const TA *act;       // gate/up: x [T][H] (bf16 calls: its f16 copy); down: h [P][I]
  const uint8_t *w;    // packed w13 or w2 (all experts)
  const float *s;      // s13 or s2
  TA *out;             // gate/up: h [P][I]; down: y [P][H]
  const float *slot_scale;  // gate/up with bf16 activations: per-slot 2^(shift - 8), else NULL
  const int *meta;
  const int4 *act_rec; // {expert, count, first slot, 0} per active expert
  const int *slot_token;
  uint32_t *status;
  // optional shared expert (same inter size): one more tile group with every
  // token, slots [P, P + T), token of slot s = s - P; expert id E marks it
  const uint8_t *sh_w;
  const float *sh_s;
  int H, I, E;
  int P, T, has_shared;
};

struct PfTile {
  int e, slot0, nvalid, npad, mt;
};

// Tile u of the call: active experts in ascending order, then the weight-row
// block, then the token tile (fastest), so CTAs working at the same time on
// one expert's token tiles share its weight stream through L2.
__device__ __forceinline__ PfTile pf_tile(int u, const int *prefix, int na, const int4 *act_rec, int MT,
                                          int na_routed, int4 shared_rec) {
  int lo = 0, hi = na - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (prefix[mid] <= u) lo = mid;
    else hi = mid - 1;
  }
  const int4 r = lo >= na_routed ? shared_rec : __ldcg(act_rec + lo);
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
// D[tmem] (+)= A[tmem] . B[smem]^T
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile("{.reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;}" ::"r"(d),
               "r"(a), "l"(b), "r"(idesc), "r"(acc));
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
// 32 lanes x 16 consecutive 32-bit columns from this warp's 16 registers per lane.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// Accumulator placement of a tile (identical in the MMA issuer and the
// epilogue): small tiles alternate between slots 0 and 1, large tiles use both.
struct PfAcc {
  uint32_t off;  // first column of gate (or first row half); second operand at off + npad
  int slot;      // 0/1 for small tiles, -1 for large ones (both slots)
};
__device__ __forceinline__ PfAcc pf_acc(int npad, int &small_count) {
  PfAcc r;
  if (npad <= kPfNSmall) {
    r.slot = small_count & 1;
    ++small_count;
    r.off = kPfAccBase + r.slot * kPfSlotCols;
  } else {
    r.slot = -1;
    r.off = kPfAccBase;
  }
  return r;
}

template <typename TA, int kMode>
__global__ void __launch_bounds__(kPfThreads, 1) k4_gemm(PfArgs<TA> a) {
  extern __shared__ __align__(1024) uint8_t pf_smem_raw[];
  uint8_t *opB = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(pf_smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t a_full[kPfAStages], a_empty[kPfAStages];
  __shared__ __align__(8) uint64_t b_full[kPfBStages], b_empty[kPfBStages];
  __shared__ __align__(8) uint64_t w_full[kPfWStages], w_empty[kPfWStages];
  __shared__ __align__(8) uint64_t acc_full[2], acc_empty[2], drain_bar;
  __shared__ int prefix[kPfMaxExperts + 2];  // active experts (+ the shared expert) + end
  __shared__ int4 tl_a[kPfMaxLocalTiles];  // {e, slot0, nvalid, npad}
  __shared__ int tl_mt[kPfMaxLocalTiles];
  __shared__ uint32_t tmem_slot;
  __shared__ volatile int abort_flag;
  __shared__ int s_na, s_na_r, s_tiles;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool gate_up = kMode == kPfGateUp;
  // f16 operands for every GEMM except the bf16 down projection
  constexpr bool kF16 = kMode == kPfGateUp || PfConv<TA>::kFmt == 0;
  constexpr uint32_t kFmt = kF16 ? 0u : 1u;
  const int kw = (kMode == kPfGateUp && PfConv<TA>::kFmt == 1) ? 8 : 0;  // weight pre-scale 2^kw
  const int K = gate_up ? a.H : a.I;                   // reduction length
  const int MT = gate_up ? a.I / 128 : a.H / 256;      // weight-row blocks per expert
  const int out_ld = gate_up ? a.I : a.H;
  const int nk = K / kPfKT;
  const int KB = K / 128;

  // ---- tile table: prefix[a] = first tile of active expert a ----
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
      s_na_r = na_r;
      s_tiles = run;
      abort_flag = 0;
    }
  }
  __syncthreads();
  const int na = s_na, na_r = s_na_r, tiles = s_tiles;
  if ((int)blockIdx.x >= tiles) return;  // CTA-uniform
  const int n_local = (tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;

  if (warp == 0) {
    for (int j = lane; j < min(n_local, kPfMaxLocalTiles); j += 32) {
      const PfTile t = pf_tile(blockIdx.x + j * gridDim.x, prefix, na, a.act_rec, MT, na_r, shared_rec);
      tl_a[j] = make_int4(t.e, t.slot0, t.nvalid, t.npad);
      tl_mt[j] = t.mt;
    }
  }
  if (tid == 0) {
    for (int s = 0; s < kPfAStages; ++s) {
      mbar_init(&a_full[s], kPfNConv * 32);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < kPfBStages; ++s) {
      mbar_init(&b_full[s], kPfNGather * 32);
      mbar_init(&b_empty[s], 1);
    }
    for (int s = 0; s < kPfWStages; ++s) {
      mbar_init(&w_full[s], 1);
      mbar_init(&w_empty[s], kPfNConv * 32);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kPfNEpi * 32);
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

  auto tile_at = [&](int j) -> PfTile {
    if (j < kPfMaxLocalTiles) {
      const int4 v = tl_a[j];
      PfTile t;
      t.e = v.x; t.slot0 = v.y; t.nvalid = v.z; t.npad = v.w; t.mt = tl_mt[j];
      return t;
    }
    return pf_tile(blockIdx.x + j * gridDim.x, prefix, na, a.act_rec, MT, na_r, shared_rec);
  };
  // Raw slice (tile t, stage kt) of weight rows: gate/up = 8 row groups x 2 KB
  // (4 chunks x gate,up x 16 rows x 16 B), down = 16 row groups x 1 KB.
  const int ngroups = gate_up ? 8 : 16;
  const uint32_t gbytes = gate_up ? 2048 : 1024;
  const size_t gstride = gate_up ? (size_t)32 * a.H : (size_t)16 * a.I;
  auto slice_src = [&](const PfTile &t, int kt) -> const uint8_t * {
    const bool sh = t.e == a.E;
    return gate_up ? (sh ? a.sh_w : a.w + (size_t)t.e * 2 * a.I * a.H) + (size_t)(t.mt * 8) * 32 * a.H +
                         (size_t)kt * 4 * 512
                   : (sh ? a.sh_w : a.w + (size_t)t.e * a.H * a.I) + (size_t)(t.mt * 16) * 16 * a.I +
                         (size_t)kt * 4 * 256;
  };

  uint8_t *wbuf = opB + kPfBStages * kPfBBytes;  // raw weight slices [kPfWStages][kPfWBytes]
  if (warp == kPfWPre) {
    // ------------------------- raw weight slices -> shared memory (TMA) ----
    // One slice = the tile's 64-column K slice of its 128 (gate, up) or 256
    // (down) weight rows: ngroups contiguous row-group pieces of the packed
    // layout, copied as they are; kPfWStages slices stay in flight.
    if (lane == 0) {
      uint32_t i = 0;
      for (int j = 0; j < n_local && !abort_flag; ++j) {
        const PfTile t = tile_at(j);
        bool ok = true;
        for (int kt = 0; kt < nk; ++kt, ++i) {
          const int ws = i % kPfWStages;
          if (!pf_wait(&w_empty[ws], ((i / kPfWStages) & 1) ^ 1, &abort_flag, a.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&w_full[ws], (uint32_t)ngroups * gbytes);
          const uint8_t *src = slice_src(t, kt);
          uint8_t *dst = wbuf + ws * kPfWBytes;
          for (int g = 0; g < ngroups; ++g) tma_bulk_g2s(dst + g * gbytes, src + g * gstride, gbytes, &w_full[ws]);
        }
        if (!ok) break;
      }
      // every issued copy lands before this CTA may exit (the converters took
      // them all unless the CTA is abandoning its work)
      for (uint32_t r = i > (uint32_t)kPfWStages ? i - kPfWStages : 0; r < i; ++r)
        if (!mbar_wait_bounded(&w_full[r % kPfWStages], (r / kPfWStages) & 1)) atomicOr(a.status, TM_STATUS_TIMEOUT);
    }
  } else if (warp == kPfWMma) {
    // ------------------------------------------------------ MMA issuer ----
    if (lane == 0) {
      uint32_t i = 0;
      uint32_t use_e[2] = {0, 0};  // acc_empty phases waited per slot
      int small_count = 0;
      bool issued = false;
      for (int j = 0; j < n_local && !abort_flag; ++j) {
        const PfTile t = tile_at(j);
        const PfAcc acc = pf_acc(t.npad, small_count);
        bool ok = true;
        for (int s = 0; s < 2 && ok; ++s)
          if (acc.slot < 0 || acc.slot == s) {
            ok = pf_wait(&acc_empty[s], (use_e[s] & 1) ^ 1, &abort_flag, a.status);
            ++use_e[s];
          }
        if (!ok) break;
        tc_fence_after();
        const uint32_t idesc = (1u << 4) | (kFmt << 7) | (kFmt << 10) | ((uint32_t)(t.npad >> 3) << 17) |
                               ((uint32_t)(128 >> 4) << 24);
        for (int kt = 0; kt < nk; ++kt, ++i) {
          const int as = i % kPfAStages, bs = i % kPfBStages;
          if (!pf_wait(&a_full[as], (i / kPfAStages) & 1, &abort_flag, a.status) ||
              !pf_wait(&b_full[bs], (i / kPfBStages) & 1, &abort_flag, a.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t bBase = smem_u32(opB + bs * kPfBBytes);
#pragma unroll
          for (int s = 0; s < kPfKT / 16; ++s) {
            const uint64_t bd = umma_desc_sw128(bBase + 32 * s);
#pragma unroll
            for (int h = 0; h < 2; ++h)
              tc_mma_ts(tmem + acc.off + h * t.npad, tmem + as * 64 + h * 32 + s * 8, bd, idesc, (kt | s) != 0);
          }
          issued = true;
          tc_commit(&a_empty[as]);
          tc_commit(&b_empty[bs]);
        }
        if (!ok) break;
        tc_commit(&acc_full[acc.slot < 0 ? 0 : acc.slot]);
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
    const int kc = gt & 7;                 // 16-byte chunk of the row's 128-byte K slice
    const int rsub = gt >> 3;              // row within each 8-row group
    // swizzled destination of (row 8q + rsub, chunk kc)
    const uint32_t dst_off = (uint32_t)rsub * 128 + (uint32_t)((kc ^ rsub) * 16);
    uint32_t i = 0;
    bool ok = true;
    for (int j = 0; j < n_local && ok && !abort_flag; ++j) {
      const PfTile t = tile_at(j);
      int rowv[kPfNMax / 8];  // source row of each of this thread's rows
#pragma unroll
      for (int q = 0; q < kPfNMax / 8; ++q) {
        const int slot = t.slot0 + min(8 * q + rsub, t.nvalid - 1);
        rowv[q] = !gate_up ? slot : slot >= a.P ? slot - a.P : __ldcg(a.slot_token + slot);
      }
      for (int kt = 0; kt < nk; ++kt, ++i) {
        const int bs = i % kPfBStages;
        if (!pf_wait(&b_empty[bs], ((i / kPfBStages) & 1) ^ 1, &abort_flag, a.status)) { ok = false; break; }
        const uint32_t dstB = smem_u32(opB + bs * kPfBBytes) + dst_off;
        const TA *base = a.act + (size_t)kt * kPfKT + kc * 8;
#pragma unroll
        for (int q = 0; q < kPfNMax / 8; ++q)
          if (8 * q < t.npad) cp_async16(dstB + q * 1024, base + (size_t)rowv[q] * K);
        cp_async_commit();
        if (i >= (uint32_t)kPfGatherLag) {
          cp_async_wait<kPfGatherLag>();
          fence_proxy_async();
          mbar_arrive(&b_full[(i - kPfGatherLag) % kPfBStages]);
        }
      }
    }
    cp_async_wait<0>();
    if (ok && !abort_flag) {
      fence_proxy_async();
      for (uint32_t r = (i > (uint32_t)kPfGatherLag ? i - kPfGatherLag : 0); r < i; ++r)
        mbar_arrive(&b_full[r % kPfBStages]);
    }
  } else if (warp < kPfWEpi) {
    // ------------------------------------------------------ converters ----
    // Thread = one weight row m (TMEM lane) of operand h: its 64-byte K slice
    // (4 chunks of 16 B) per stage, read from the raw slice the producer warp
    // staged in shared memory (16 consecutive lanes read 256 contiguous bytes:
    // no bank conflicts).  The block scales run two slices ahead in registers.
    const int h = (warp - kPfWConv) >> 2;
    const int q = warp & 3;
    const int m = q * 32 + lane;
    const uint32_t tlane = tmem + ((uint32_t)(q * 32) << 16);
    // byte offset of (row m of operand h, chunk 0) inside a staged slice; chunk stride
    const int row_off = gate_up ? (m >> 4) * 2048 + h * 256 + (m & 15) * 16 : (h * 8 + (m >> 4)) * 1024 + (m & 15) * 16;
    const int cstride = gate_up ? 512 : 256;
    auto scale_ptr = [&](const PfTile &t) -> const float * {
      if (t.e == a.E)
        return gate_up ? a.sh_s + ((size_t)t.mt * 2 + h) * KB : a.sh_s + ((size_t)t.mt * 2 + h) * (a.I / 128);
      return gate_up ? a.s + ((size_t)(t.e * (a.I / 128) + t.mt) * 2 + h) * KB
                     : a.s + ((size_t)t.e * (a.H / 128) + t.mt * 2 + h) * (a.I / 128);
    };
    int pj = 0, pkt = 0;  // next slice whose scale to load
    PfTile pt = tile_at(0);
    auto load_scale = [&](float &sc) {
      sc = __ldg(scale_ptr(pt) + (pkt * kPfKT) / 128);
      if (++pkt == nk) {
        pkt = 0;
        if (++pj < n_local) pt = tile_at(pj);
      }
    };
    const uint32_t total = (uint32_t)n_local * (uint32_t)nk;
    float s0 = 0.f, s1 = 0.f, s2 = 0.f;
    load_scale(s0);
    if (total > 1) load_scale(s1);
    for (uint32_t i = 0; i < total && !abort_flag; ++i) {
      if (i + 2 < total) load_scale(s2);
      const int wsi = i % kPfWStages;
      if (!__all_sync(0xffffffffu, pf_wait(&w_full[wsi], (i / kPfWStages) & 1, &abort_flag, a.status))) break;
      uint4 b0[4];
      const uint8_t *wsrc = wbuf + wsi * kPfWBytes + row_off;
#pragma unroll
      for (int c = 0; c < 4; ++c) b0[c] = *reinterpret_cast<const uint4 *>(wsrc + c * cstride);
      // dequantise while the A stage may still be read by the MMAs of slice i - kPfAStages
      uint32_t wv[2][16];
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // chunks 2*half, 2*half + 1 -> 16 TMEM columns
#pragma unroll
        for (int cc = 0; cc < 2; ++cc) {
          const uint4 v = b0[2 * half + cc];
          uint32_t *w = wv[half];
          if constexpr (kF16) {
            const uint32_t S = pf_scale_f16(s0, kw);
            pf_convert4_f16(v.x, S, w[8 * cc + 0], w[8 * cc + 1]);
            pf_convert4_f16(v.y, S, w[8 * cc + 2], w[8 * cc + 3]);
            pf_convert4_f16(v.z, S, w[8 * cc + 4], w[8 * cc + 5]);
            pf_convert4_f16(v.w, S, w[8 * cc + 6], w[8 * cc + 7]);
          } else {
            const uint32_t S = PfConv<TA>::scale(s0);
            pf_convert4_bf16(v.x, S, w[8 * cc + 0], w[8 * cc + 1]);
            pf_convert4_bf16(v.y, S, w[8 * cc + 2], w[8 * cc + 3]);
            pf_convert4_bf16(v.z, S, w[8 * cc + 4], w[8 * cc + 5]);
            pf_convert4_bf16(v.w, S, w[8 * cc + 6], w[8 * cc + 7]);
          }
        }
      }
      mbar_arrive(&w_empty[wsi]);  // the slice's bytes are in registers
      const int as = i % kPfAStages;
      // warp-uniform outcome: the tcgen05.st below is .sync.aligned
      if (!__all_sync(0xffffffffu, pf_wait(&a_empty[as], ((i / kPfAStages) & 1) ^ 1, &abort_flag, a.status))) break;
      tc_fence_after();
      tc_st16(tlane + as * 64 + h * 32, wv[0]);
      tc_st16(tlane + as * 64 + h * 32 + 16, wv[1]);
      tc_wait_st();
      tc_fence_before();
      mbar_arrive(&a_full[as]);
      s0 = s1;
      s1 = s2;
    }
  } else {
    // -------------------------------------------------------- epilogue ----
    // two warps per TMEM lane quadrant; warp half `hf` takes the 16-column
    // chunks 2c + hf of every tile
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int hf = (warp - kPfWEpi) >> 2;
    const int m = q * 32 + lane;
    uint32_t use_f[2] = {0, 0};
    int small_count = 0;
    for (int j = 0; j < n_local && !abort_flag; ++j) {
      const PfTile t = tile_at(j);
      const PfAcc acc = pf_acc(t.npad, small_count);
      const int fs = acc.slot < 0 ? 0 : acc.slot;
      // warp-uniform outcome: the tcgen05.ld below is .sync.aligned
      if (!__all_sync(0xffffffffu, pf_wait(&acc_full[fs], use_f[fs] & 1, &abort_flag, a.status))) break;
      ++use_f[fs];
      tc_fence_after();
      const uint32_t tb = tmem + ((uint32_t)(q * 32) << 16) + acc.off;
      // column scales (undo the token's f16 shift and the weights' 2^kw; exact
      // powers of 2): lane jj of the warp holds the scale of column c0 + jj,
      // loaded one chunk ahead
      auto col_scale = [&](int c0) -> float {
        return (a.slot_scale && lane < 16 && c0 + lane < t.nvalid) ? __ldcg(a.slot_scale + t.slot0 + c0 + lane) : 1.f;
      };
      float cs_next = gate_up ? col_scale(16 * hf) : 1.f;
      for (int c0 = 16 * hf; c0 < t.nvalid; c0 += 32) {
        const float cs_cur = cs_next;
        if (gate_up && c0 + 32 < t.nvalid) cs_next = col_scale(c0 + 32);
        float v0[16], v1[16];
        // the registers of an asynchronous TMEM load are read only after the
        // wait, with nothing in between (their values land later)
        tc_ld16(tb + c0, v0);
        tc_ld16(tb + t.npad + c0, v1);
        tc_wait_ld();
        if (gate_up) {
          TA *o = a.out + (size_t)(t.slot0 + c0) * out_ld + t.mt * 128 + m;
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const float cs = __shfl_sync(0xffffffffu, cs_cur, jj);
            if (c0 + jj < t.nvalid) {
              const float g = v0[jj] * cs, u = v1[jj] * cs;
              o[(size_t)jj * out_ld] = Act<TA>::from_f(__fdividef(g, 1.0f + __expf(-g)) * u);
            }
          }
        } else {
          TA *o = a.out + (size_t)(t.slot0 + c0) * out_ld + t.mt * 256 + m;
#pragma unroll
          for (int jj = 0; jj < 16; ++jj)
            if (c0 + jj < t.nvalid) {
              o[(size_t)jj * out_ld] = Act<TA>::from_f(v0[jj]);
              o[(size_t)jj * out_ld + 128] = Act<TA>::from_f(v1[jj]);
            }
        }
      }
      tc_fence_before();
      for (int s = 0; s < 2; ++s)
        if (acc.slot < 0 || acc.slot == s) mbar_arrive(&acc_empty[s]);
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
constexpr int kPfMaxTopK = 64;  // combine: slot ids and weights of one token in shared memory

// out[t] = sum_r w[t,r] * y[slot(t,r)] (top-k order, fp32) (+ gated shared
// expert) (+ residual), rounded once.  One CTA per token; each thread owns 8
// columns and issues its loads of up to 8 ranks before accumulating them.
template <typename TA>
__global__ void __launch_bounds__(256) k4_combine(const TA *y, const TA *w, const int *pair_slot, const TA *residual,
                                                  TA *out, int H, int k, const float *sh_w, int sh_slot0) {
  __shared__ int s_slot[kPfMaxTopK];
  __shared__ float s_w[kPfMaxTopK];
  const int t = blockIdx.x;
  for (int r = threadIdx.x; r < k; r += blockDim.x) {
    s_slot[r] = __ldcg(pair_slot + (size_t)t * k + r);
    s_w[r] = Act<TA>::to_f(w[(size_t)t * k + r]);
  }
  __syncthreads();
  for (int o = threadIdx.x * 8; o < H; o += blockDim.x * 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r0 = 0; r0 < k; r0 += 8) {
      uint4 v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int r = r0 + u;
        const int sl = r < k ? s_slot[r] : -1;
        v[u] = sl >= 0 ? __ldcg(reinterpret_cast<const uint4 *>(y + (size_t)sl * H + o)) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int r = r0 + u;
        if (r < k && s_slot[r] >= 0) {
          const float wr = s_w[r];
          const TA *yv = reinterpret_cast<const TA *>(&v[u]);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = fmaf(wr, Act<TA>::to_f(yv[j]), acc[j]);
        }
      }
    }
    if (sh_w) {  // gated shared expert (moe.py:200): after the routed sum
      const float ws = __ldcg(sh_w + t);
      const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(y + (size_t)(sh_slot0 + t) * H + o));
      const TA *yv = reinterpret_cast<const TA *>(&v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = fmaf(ws, Act<TA>::to_f(yv[j]), acc[j]);
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

// Per token, one warp (8 tokens per CTA; a row of up to 2048 16-bit values
// stays in the lane's registers between the two passes):
//  * bf16 activations (x16 != NULL): x[t] -> f16 x16[t] = x[t] * 2^-s_t with
//    s_t from the row's max |x| (exact for bf16 values: 8 significant bits into
//    f16's 11, the row maximum scaled into [2^13, 2^14)), and for each of the
//    token's slots (its k routed ones and, with a shared expert, slot
//    sh_slot0 + t) slot_scale = 2^(s_t - 8), which undoes the shift and the
//    weights' 2^8 in the gate/up epilogue;
//  * with a shared expert (sh_gate_w != NULL): its gate score
//    sh_w[t] = sigmoid(x[t] . sh_gate_w), F.linear's output and the sigmoid
//    each rounded to the act dtype (moe.py:196-198).
constexpr int kPrepWarps = 8;
constexpr int kPrepVecs = 8;  // 16-byte vectors per lane kept in registers
template <typename TA>
__global__ void __launch_bounds__(kPrepWarps * 32) k4_prep(const TA *x, const int *pair_slot, int T, int H, int k,
                                                           __half *x16, float *slot_scale, const TA *sh_gate_w,
                                                           float *sh_w, int sh_slot0) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kPrepWarps + (threadIdx.x >> 5);
  if (t >= T) return;  // warp-uniform
  int used = sh_gate_w != nullptr;
  for (int r = lane; r < k && !used; r += 32) used = __ldcg(pair_slot + (size_t)t * k + r) >= 0;
  if (!__any_sync(0xffffffffu, used)) return;  // a row no slot reads (capacity rows of an expert-parallel owner)
  const uint4 *xr = reinterpret_cast<const uint4 *>(x + (size_t)t * H);
  const uint4 *gr = reinterpret_cast<const uint4 *>(sh_gate_w);
  const int nv = H / 8;
  float m = 0.f, gl = 0.f;
  uint4 keep[kPrepVecs];
  for (int b = 0; b < nv; b += 32 * kPrepVecs) {
#pragma unroll
    for (int u = 0; u < kPrepVecs; ++u) {
      const int i = b + u * 32 + lane;
      if (i < nv) {
        const uint4 v = __ldcg(xr + i);
        if (b == 0) keep[u] = v;
        const TA *p = reinterpret_cast<const TA *>(&v);
        if (sh_gate_w) {
          const uint4 gv = __ldg(gr + i);
          const TA *gp = reinterpret_cast<const TA *>(&gv);
#pragma unroll
          for (int j = 0; j < 8; ++j) gl = fmaf(Act<TA>::to_f(p[j]), Act<TA>::to_f(gp[j]), gl);
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) m = fmaxf(m, fabsf(Act<TA>::to_f(p[j])));
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    gl += __shfl_xor_sync(0xffffffffu, gl, o);
  }
  if (sh_gate_w && lane == 0) {
    const float logit = Act<TA>::round(gl);
    sh_w[t] = Act<TA>::round(1.0f / (1.0f + __expf(-logit)));
  }
  if (!x16) return;
  const int sh = f16_shift(m);
  for (int b = 0; b < nv; b += 32 * kPrepVecs) {
#pragma unroll
    for (int u = 0; u < kPrepVecs; ++u) {
      const int i = b + u * 32 + lane;
      if (i < nv) {
        const uint4 v = b == 0 ? keep[u] : __ldcg(xr + i);
        const TA *p = reinterpret_cast<const TA *>(&v);
        uint4 r;
        __half *q = reinterpret_cast<__half *>(&r);
#pragma unroll
        for (int j = 0; j < 8; ++j) q[j] = __float2half_rn(ldexpf(Act<TA>::to_f(p[j]), -sh));
        reinterpret_cast<uint4 *>(x16 + (size_t)t * H)[i] = r;
      }
    }
  }
  const float scale = ldexpf(1.f, sh - 8);
  for (int r = lane; r < k; r += 32) {
    const int sl = __ldcg(pair_slot + (size_t)t * k + r);
    if (sl >= 0) slot_scale[sl] = scale;
  }
  if (sh_gate_w && lane == 0) slot_scale[sh_slot0 + t] = scale;
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
  bool combine;  // false: stop after the down GEMM (per-slot outputs in the ypart region)
  // optional shared expert (inter size I): packed weights and the gate row [H]
  const uint8_t *sh_w13; const float *sh_s13; const uint8_t *sh_w2; const float *sh_s2; const void *sh_gate_w;
  template <typename TA> int run() {
    if constexpr (sizeof(TA) != 2) {
      return fail(TM_ERR_UNSUPPORTED, "tm_moe_prefill_grouped: fp32 activations are not supported (bf16, fp16)");
    } else {
      const bool shared = sh_w13 != nullptr;
      const int64_t P = T * k;
      PfArgs<TA> g;
      g.meta = ws_ptr<int>(ws, L->meta);
      g.act_rec = ws_ptr<int4>(ws, L->act_rec);
      g.slot_token = ws_ptr<int>(ws, L->slot_token);
      g.status = ws_ptr<uint32_t>(ws, L->status);
      g.H = H; g.I = I; g.E = E;
      g.P = (int)P; g.T = (int)T; g.has_shared = shared ? 1 : 0;
      g.sh_w = sh_w13; g.sh_s = sh_s13;
      // slots: routed [0, P), shared [P, P + T)
      TA *h = ws_ptr<TA>(ws, L->h);        // [P (+T)][I] act dtype (region sized for P x I fp32)
      TA *y = ws_ptr<TA>(ws, L->ypart);    // [P (+T)][H] act dtype (region sized for (P + T) x H fp32)
      float *sh_w = ws_ptr<float>(ws, L->sh_w);  // [T]
      const int grid = num_sms();
      g.act = (const TA *)x; g.w = w13; g.s = s13; g.out = h; g.slot_scale = nullptr;
      if constexpr (PfConv<TA>::kFmt == 1) {
        // bf16: the gate/up GEMM runs on f16 operands (x16 after the slots' outputs in the ypart region)
        __half *x16 = reinterpret_cast<__half *>(reinterpret_cast<char *>(y) + (size_t)(P + T) * H * sizeof(TA));
        float *slot_scale = ws_ptr<float>(ws, L->logits);  // [P + T] (the region holds T * E floats)
        k4_prep<TA><<<(unsigned)((T + kPrepWarps - 1) / kPrepWarps), kPrepWarps * 32, 0, s>>>(
            (const TA *)x, ws_ptr<int>(ws, L->pair_slot), (int)T, H, k, x16, slot_scale,
                                                shared ? (const TA *)sh_gate_w : nullptr, sh_w, (int)P);
        TM_LAUNCH_CHECK("k4_prep launch");
        g.act = (const TA *)x16;
        g.slot_scale = slot_scale;
      } else if (shared) {
        k4_prep<TA><<<(unsigned)((T + kPrepWarps - 1) / kPrepWarps), kPrepWarps * 32, 0, s>>>(
            (const TA *)x, ws_ptr<int>(ws, L->pair_slot), (int)T, H, k, nullptr, nullptr,
                                                (const TA *)sh_gate_w, sh_w, (int)P);
        TM_LAUNCH_CHECK("k4_prep launch");
      }
      int rc = ensure_smem(reinterpret_cast<const void *>(k4_gemm<TA, kPfGateUp>), kPfSmem);
      if (rc) return rc;
      k4_gemm<TA, kPfGateUp><<<grid, kPfThreads, kPfSmem, s>>>(g);
      TM_LAUNCH_CHECK("k4_gemm gate/up launch");
      g.act = h; g.w = w2; g.s = s2; g.out = y; g.slot_scale = nullptr;
      g.sh_w = sh_w2; g.sh_s = sh_s2;
      rc = ensure_smem(reinterpret_cast<const void *>(k4_gemm<TA, kPfDown>), kPfSmem);
      if (rc) return rc;
      k4_gemm<TA, kPfDown><<<grid, kPfThreads, kPfSmem, s>>>(g);
      TM_LAUNCH_CHECK("k4_gemm down launch");
      if (!combine) return TM_OK;
      k4_combine<TA><<<(unsigned)T, 256, 0, s>>>(y, (const TA *)topk_w, ws_ptr<int>(ws, L->pair_slot),
                                                   (const TA *)residual, (TA *)out, H, k,
                                                   shared ? sh_w : nullptr, (int)P);
      TM_LAUNCH_CHECK("k4_combine launch");
      return TM_OK;
    }
  }
};

}  // namespace tmoe

using namespace tmoe;

namespace tmoe {
struct CombineLaunch {
  const void *y; const void *w; const int *pair_slot; const void *residual; void *out; int64_t T; int H, k;
  cudaStream_t s;
  template <typename TA> int run() {
    if constexpr (sizeof(TA) != 2) {
      return fail(TM_ERR_UNSUPPORTED, "tm_combine_slots: act dtype must be bf16 or fp16");
    } else {
      k4_combine<TA><<<(unsigned)T, 256, 0, s>>>((const TA *)y, (const TA *)w, pair_slot, (const TA *)residual,
                                                   (TA *)out, H, k, nullptr, 0);
      TM_LAUNCH_CHECK("k4_combine launch");
      return TM_OK;
    }
  }
};
}  // namespace tmoe

namespace tmoe {
struct CombineAllLaunch {
  const void *y; const void *w; const int *pair_slot; const void *residual; void *out; int64_t T; int H, k;
  const float *sh_w; int sh_slot0; cudaStream_t s;
  template <typename TA> int run() {
    if constexpr (sizeof(TA) != 2) {
      return fail(TM_ERR_UNSUPPORTED, "combine: act dtype must be bf16 or fp16");
    } else {
      k4_combine<TA><<<(unsigned)T, 256, 0, s>>>((const TA *)y, (const TA *)w, pair_slot, (const TA *)residual,
                                                   (TA *)out, H, k, sh_w, sh_slot0);
      TM_LAUNCH_CHECK("k4_combine launch");
      return TM_OK;
    }
  }
};
int combine_expert_outputs(const void *y, const void *topk_w, const int *pair_slot, const void *residual, void *out,
                           int64_t T, int H, int k, int act_dtype, const float *sh_w, int sh_slot0, cudaStream_t s) {
  TM_REQUIRE(k >= 1 && k <= kPfMaxTopK && H % 8 == 0, "combine: bad shape");
  CombineAllLaunch f{y, topk_w, pair_slot, residual, out, T, H, k, sh_w, sh_slot0, s};
  return dispatch_act(act_dtype, f);
}
}  // namespace tmoe

extern "C" int tm_combine_slots(const void *y, const void *topk_w, const int32_t *pair_slot, int64_t tokens,
                                int hidden, int top_k, int act_dtype, const void *residual, void *out,
                                void *stream) {
  TM_REQUIRE(y && topk_w && pair_slot && out, "null pointer");
  TM_REQUIRE(tokens >= 1 && top_k >= 1 && top_k <= kPfMaxTopK && hidden > 0 && hidden % 8 == 0, "bad shape");
  TM_REQUIRE(aligned(y, 16) && aligned(out, 16) && (!residual || aligned(residual, 16)),
             "y, residual and out must be 16-byte aligned");
  CombineLaunch f{y, topk_w, pair_slot, residual, out, tokens, hidden, top_k, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_moe_prefill_grouped(const void *x, int64_t tokens, int hidden, int inter, int n_experts,
                                      int top_k, int act_dtype, const void *topk_w, const uint8_t *w13,
                                      const float *s13, const uint8_t *w2, const float *s2, const uint8_t *sh_w13,
                                      const float *sh_s13, const uint8_t *sh_w2, const float *sh_s2,
                                      int shared_inter, const void *sh_gate_w, const void *residual, void *out,
                                      void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(x && topk_w && w13 && s13 && w2 && s2 && out, "null pointer");
  const bool shared = sh_w13 != nullptr;
  TM_REQUIRE(!shared || (sh_s13 && sh_w2 && sh_s2 && sh_gate_w), "shared expert: every pointer or none");
  if (shared) {
    TM_REQUIRE(shared_inter == inter, "shared expert inter %d != inter %d (the grouped GEMMs need one size)",
               shared_inter, inter);
    TM_REQUIRE(n_experts > top_k, "shared expert needs n_experts > top_k (slot scale region)");
    TM_REQUIRE(aligned(sh_w13, 16) && aligned(sh_w2, 16) && aligned(sh_gate_w, 16),
               "shared weights must be 16-byte aligned");
  }
  TM_REQUIRE(hidden % 256 == 0 && hidden > 0 && hidden <= 128 * kPfMaxKBlocks,
             "hidden (%d) must be a positive multiple of 256, at most %d", hidden, 128 * kPfMaxKBlocks);
  TM_REQUIRE(inter % 128 == 0 && inter > 0 && inter <= 128 * kPfMaxKBlocks,
             "inter (%d) must be a positive multiple of 128, at most %d", inter, 128 * kPfMaxKBlocks);
  TM_REQUIRE(n_experts <= kPfMaxExperts, "n_experts %d > %d", n_experts, kPfMaxExperts);
  TM_REQUIRE(top_k >= 1 && top_k <= kPfMaxTopK, "top_k %d outside [1, %d]", top_k, kPfMaxTopK);
  TM_REQUIRE(aligned(x, 16) && aligned(w13, 16) && aligned(w2, 16) && aligned(out, 16) &&
                 (!residual || aligned(residual, 16)),
             "x, weights, residual and out must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, inter, shared ? shared_inter : 0, &L);
  if (rc) return rc;
  PrefillLaunch f{x, tokens, hidden, inter, n_experts, top_k, topk_w, w13, s13, w2, s2, residual, out,
                  ws, &L, as_stream(stream), true};
  if (shared) {
    f.sh_w13 = sh_w13; f.sh_s13 = sh_s13; f.sh_w2 = sh_w2; f.sh_s2 = sh_s2; f.sh_gate_w = sh_gate_w;
  }
  return dispatch_act(act_dtype, f);
}

namespace tmoe {
int prefill_expert_outputs(const void *x, int64_t tokens, int hidden, int inter, int n_experts, int top_k,
                           int act_dtype, const uint8_t *w13, const float *s13, const uint8_t *w2, const float *s2,
                           void *ws, const WsLayout &L, cudaStream_t stream) {
  TM_REQUIRE(hidden % 256 == 0 && hidden > 0 && hidden <= 128 * kPfMaxKBlocks, "hidden (%d) unsupported", hidden);
  TM_REQUIRE(inter % 128 == 0 && inter > 0 && inter <= 128 * kPfMaxKBlocks, "inter (%d) unsupported", inter);
  TM_REQUIRE(n_experts <= kPfMaxExperts, "n_experts %d > %d", n_experts, kPfMaxExperts);
  PrefillLaunch f{x, tokens, hidden, inter, n_experts, top_k, nullptr, w13, s13, w2, s2, nullptr, nullptr,
                  ws, &L, stream, false, nullptr, nullptr, nullptr, nullptr, nullptr};
  return dispatch_act(act_dtype, f);
}
}  // namespace tmoe

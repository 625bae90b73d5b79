// K1: fused router (logits GEMV + fp32 softmax + top-k + renormalisation) and
// the routing plan (histogram, offsets, active experts, stable permutation).
//
// Reference: RouterExecutor.compute_routing (execution/router.py:15-42) and the
// implicit grouping in MoEExecutor.execute_layer (execution/moe.py:132,164-165):
// experts ascending (torch.unique), tokens ascending within an expert
// (torch.where over [T, k] in row-major order).
//
// Latency matters more than bandwidth here (one decode layer reads 0.5 MB of
// router weights): each warp holds its expert row in registers before
// griddepcontrol.wait (weights do not depend on the previous kernel), the
// token tile arrives by one TMA bulk copy, and no loop carries a chain of
// dependent global loads.
#include <cooperative_groups.h>

#include "tm_common.cuh"

namespace cg = cooperative_groups;

namespace tmoe {

constexpr int kRouterThreads = 256;     // 8 warps
constexpr int kRouterWarps = kRouterThreads / 32;
constexpr int kMaxExpertsPerLane = 32;  // E <= 1024
constexpr int kRowVecs = 16;            // 16-byte vectors of a router row a lane keeps in registers
constexpr int kClusterCTAs = 8;         // decode router: one thread-block cluster
constexpr int kClusterMaxE = kClusterCTAs * kRouterWarps * 2;  // 2 expert rows per warp
constexpr int kClusterMaxT = 8;
constexpr int kClusterMaxTFast = 2;  // beyond this the tensor-core router is faster (measured on B200)

struct PlanPtrs {
  uint32_t *status;
  uint32_t *trace;  // trace builds only
  int *meta;
  int *counts;    // [E]
  int *offsets;   // [E+1]
  int *act_list;  // [E]
  int4 *act_rec;  // [E]
  int *slot_token, *slot_pair, *pair_slot;  // [P]
  int *k2_cnt;    // [(E+1)*kMaxRG]
  int *k3_cnt;    // [kMaxRGo]
  int *unit_hist; // [ceil(T/16)][E]
  int k2_cnt_n, k3_cnt_n;
};

static PlanPtrs plan_ptrs(void *ws, const WsLayout &L) {
  PlanPtrs p;
  p.status = ws_ptr<uint32_t>(ws, L.status);
  p.trace = kTraceBytes ? ws_ptr<uint32_t>(ws, L.trace) : nullptr;
  p.meta = ws_ptr<int>(ws, L.meta);
  p.counts = ws_ptr<int>(ws, L.counts);
  p.offsets = ws_ptr<int>(ws, L.offsets);
  p.act_list = ws_ptr<int>(ws, L.act_list);
  p.act_rec = ws_ptr<int4>(ws, L.act_rec);
  p.slot_token = ws_ptr<int>(ws, L.slot_token);
  p.slot_pair = ws_ptr<int>(ws, L.slot_pair);
  p.pair_slot = ws_ptr<int>(ws, L.pair_slot);
  p.k2_cnt = ws_ptr<int>(ws, L.k2_cnt);
  p.k3_cnt = ws_ptr<int>(ws, L.k3_cnt);
  p.unit_hist = ws_ptr<int>(ws, L.unit_hist);
  p.k2_cnt_n = 0;  // K2 keeps no counters
  p.k3_cnt_n = kMaxRGo;
  return p;
}

// In-place exclusive scan of a[0..n) by the whole block; returns the total.
// `tmp` needs 33 ints of shared memory.
__device__ int block_excl_scan(int *a, int n, int *tmp) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, w = tid >> 5, nw = nt >> 5;
  const int seg = (n + nt - 1) / nt;
  const int lo = min(n, tid * seg), hi = min(n, lo + seg);
  int local = 0;
  for (int i = lo; i < hi; ++i) local += a[i];
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) tmp[w] = incl;
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int i = 0; i < nw; ++i) {
      int c = tmp[i];
      tmp[i] = run;
      run += c;
    }
    tmp[32] = run;
  }
  __syncthreads();
  int run = tmp[w] + incl - local;
  for (int i = lo; i < hi; ++i) {
    int c = a[i];
    a[i] = run;
    run += c;
  }
  __syncthreads();
  int total = tmp[32];
  __syncthreads();
  return total;
}

// In-place exclusive scans of a[0..n) and b[0..n) by the whole block in one
// pass (warp totals scanned by one warp); returns both totals.  tmp holds at
// least 66 ints.
__device__ int2 block_excl_scan2(int *a, int *b, int n, int *tmp) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, w = tid >> 5, nw = nt >> 5;
  const int seg = (n + nt - 1) / nt;
  const int lo = min(n, tid * seg), hi = min(n, lo + seg);
  int la = 0, lb = 0;
  for (int i = lo; i < hi; ++i) {
    la += a[i];
    lb += b[i];
  }
  int ia = la, ib = lb;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int va = __shfl_up_sync(0xffffffffu, ia, o), vb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += va;
      ib += vb;
    }
  }
  if (lane == 31) {
    tmp[w] = ia;
    tmp[32 + w] = ib;
  }
  __syncthreads();
  if (w == 0) {
    const int xa = lane < nw ? tmp[lane] : 0, xb = lane < nw ? tmp[32 + lane] : 0;
    int sa = xa, sb = xb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int va = __shfl_up_sync(0xffffffffu, sa, o), vb = __shfl_up_sync(0xffffffffu, sb, o);
      if (lane >= o) {
        sa += va;
        sb += vb;
      }
    }
    if (lane < nw) {
      tmp[lane] = sa - xa;
      tmp[32 + lane] = sb - xb;
    }
    if (lane == 31) {
      tmp[64] = sa;
      tmp[65] = sb;
    }
  }
  __syncthreads();
  int ra = tmp[w] + ia - la, rb = tmp[32 + w] + ib - lb;
  for (int i = lo; i < hi; ++i) {
    const int ca = a[i], cb = b[i];
    a[i] = ra;
    b[i] = rb;
    ra += ca;
    rb += cb;
  }
  const int2 tot = make_int2(tmp[64], tmp[65]);
  __syncthreads();
  return tot;
}

// Top-k index of pair p: from shared memory when this CTA selected them, else
// (written by other CTAs of the grid, or by the caller) from global memory.
struct IdxSource {
  const int64_t *g;
  const int *s;
  __device__ __forceinline__ int64_t get(int p) const { return s ? (int64_t)s[p] : __ldcg(g + p); }
};

// Build the routing plan from the [T, k] top-k indices.  Whole block; `sm`
// needs (nwarps * E + 3 * E + 64) ints of shared memory.
__device__ void plan_build(IdxSource idx, int T, int k, int E, const PlanPtrs &pp, int *sm) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, nw = blockDim.x >> 5;
  const int P = T * k;
  int *hist = sm;                    // [nw][E]
  int *cnt = sm + nw * E;            // [E] counts, then offsets
  int *flag = cnt + E;               // [E] active flag, then active index
  int *cnt0 = flag + E;              // [E] counts (kept)
  int *tmp = cnt0 + E;               // [33]
  for (int i = tid; i < nw * E; i += blockDim.x) hist[i] = 0;
  // the expert kernels' completion counters are zeroed for this call
  for (int i = tid; i < pp.k2_cnt_n; i += blockDim.x) pp.k2_cnt[i] = 0;
  for (int i = tid; i < pp.k3_cnt_n; i += blockDim.x) pp.k3_cnt[i] = 0;
  __syncthreads();
  const int lo = (int)((int64_t)w * P / nw), hi = (int)((int64_t)(w + 1) * P / nw);
  bool bad = false;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    if (p < hi) {
      const int64_t e = idx.get(p);
      if (e >= 0 && e < E) atomicAdd(&hist[w * E + (int)e], 1);
      else bad = true;
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(pp.status, TM_STATUS_BAD_EXPERT_ID);
  __syncthreads();
  // per expert: exclusive prefix over warps, total count
  for (int e = tid; e < E; e += blockDim.x) {
    int run = 0;
    for (int j = 0; j < nw; ++j) {
      int c = hist[j * E + e];
      hist[j * E + e] = run;
      run += c;
    }
    cnt[e] = run;
    cnt0[e] = run;
    flag[e] = run > 0 ? 1 : 0;
    pp.counts[e] = run;
  }
  __syncthreads();
  const int total = block_excl_scan(cnt, E, tmp);
  const int n_active = block_excl_scan(flag, E, tmp);
  for (int e = tid; e < E; e += blockDim.x) {
    const int c = cnt0[e];
    pp.offsets[e] = cnt[e];
    if (c > 0) {
      pp.act_list[flag[e]] = e;
      pp.act_rec[flag[e]] = make_int4(e, c, cnt[e], 0);
    }
    for (int j = 0; j < nw; ++j) hist[j * E + e] += cnt[e];
  }
  if (tid == 0) {
    pp.offsets[E] = total;
    pp.meta[kMetaNActive] = n_active;
    pp.meta[kMetaPairs] = P;
    pp.meta[kMetaTokens] = T;
  }
  __syncthreads();
  // stable scatter: pairs of warp w's range, in order, 32 at a time
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    int e = -1;
    if (p < hi) {
      const int64_t v = idx.get(p);
      e = (v >= 0 && v < E) ? (int)v : -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt_mask);
    if (p < hi) {
      if (e >= 0) {
        const int slot = hist[w * E + e] + rank;
        pp.slot_pair[slot] = p;
        pp.slot_token[slot] = p / k;
        pp.pair_slot[p] = slot;
      } else {
        pp.pair_slot[p] = -1;
      }
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) hist[w * E + e] += __popc(peers);
    __syncwarp();
  }
}

template <typename TA> struct RouterArgs {
  const TA *x;
  const TA *w;
  int64_t *idx_out;
  TA *w_out;
  TA *logits_out;
  float *logits_ws;
  int *tile_cnt;   // [kMaxTokenTiles] + done counter at [kMaxTokenTiles]
  int T, H, E, k;
  int TB;          // tokens per token tile
  int EPW;         // experts per warp per CTA
  int n_etiles, n_ttiles;
  PlanPtrs pp;
  // one-token router only (NULL: none): x is first RMS-normalised with this
  // weight (Qwen3MoeRMSNorm, k8_rmsnorm's arithmetic), the routing uses the
  // normalised token, and CTA 0 writes it to x_norm_out for the expert kernels
  const TA *norm_w;
  float eps;
  TA *x_norm_out;
};

// Routing plan of a call with at most 32 (token, rank) pairs: one warp,
// registers and a few shared words, no block-wide barrier.  Same result as
// plan_build.  The caller's other warps zero the expert kernels' counters.
__device__ void plan_small_warp(IdxSource idx, int T, int k, int E, const PlanPtrs &pp) {
  __shared__ int s_ae[32], s_ac[32];
  const int lane = threadIdx.x & 31;
  const int P = T * k;
  int e = -1;
  if (lane < P) {
    const int64_t v = idx.get(lane);
    e = (v >= 0 && v < E) ? (int)v : -1;
  }
  if (__any_sync(0xffffffffu, lane < P && e < 0) && lane == 0) atomicOr(pp.status, TM_STATUS_BAD_EXPERT_ID);
  const unsigned peers = __match_any_sync(0xffffffffu, e);
  const bool leader = e >= 0 && lane == __ffs(peers) - 1;
  const unsigned leaders = __ballot_sync(0xffffffffu, leader);
  int less = 0, act = 0;  // valid pairs / distinct experts with a smaller expert id
  for (int q = 0; q < 32; ++q) {
    const int eq = __shfl_sync(0xffffffffu, e, q);
    less += (eq >= 0 && eq < e);
    act += ((leaders >> q) & 1u) && eq < e;
  }
  const int n_active = __popc(leaders);
  if (lane < P) {
    if (e >= 0) {
      const int slot = less + __popc(peers & ((1u << lane) - 1u));
      pp.slot_pair[slot] = lane;
      pp.slot_token[slot] = lane / k;
      pp.pair_slot[lane] = slot;
    } else {
      pp.pair_slot[lane] = -1;
    }
  }
  if (leader) {
    pp.act_list[act] = e;
    pp.act_rec[act] = make_int4(e, __popc(peers), less, 0);
    s_ae[act] = e;
    s_ac[act] = __popc(peers);
  }
  __syncwarp();
  for (int x = lane; x <= E; x += 32) {
    int below = 0, cnt = 0;
    for (int a = 0; a < n_active; ++a) {
      below += s_ae[a] < x ? s_ac[a] : 0;
      cnt += s_ae[a] == x ? s_ac[a] : 0;
    }
    pp.offsets[x] = below;
    if (x < E) pp.counts[x] = cnt;
  }
  if (lane == 0) {
    pp.meta[kMetaNActive] = n_active;
    pp.meta[kMetaPairs] = P;
    pp.meta[kMetaTokens] = T;
  }
}

// softmax(fp32) + top-k (value desc, lower id first on ties) + renormalise, one
// warp per token, EPL = experts per lane (compile time: compact code).  Lane r
// keeps the r-th winner; all lanes write in parallel.
template <typename TA, int EPL>
__device__ void router_topk_token(const RouterArgs<TA> &a, int t, int *s_idx) {
  const int lane = threadIdx.x & 31;
  const float *lg = a.logits_ws + (int64_t)t * a.E;
  float v[EPL];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < a.E ? ld_cg(lg + e) : -INFINITY;
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i)
    if (i * 32 + lane < a.E) s += __expf(v[i] - m);
  s = warp_sum(s);
  unsigned taken = 0;  // bit i: v[i] already selected
  float my_p = 0.f, psum = 0.f;
  int my_e = 0;
  for (int r = 0; r < a.k; ++r) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = i * 32 + lane;
      if (e < a.E && !(taken & (1u << i))) {
        if (v[i] > bv || (v[i] == bv && e < be)) { bv = v[i]; be = e; }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) { bv = ov; be = oe; }
    }
    if ((be & 31) == lane) taken |= 1u << (be >> 5);
    const float p = __expf(bv - m) / s;  // softmax probability of the winner
    psum += p;
    if (lane == r) { my_e = be; my_p = p; }
  }
  if (lane < a.k) {
    a.idx_out[(int64_t)t * a.k + lane] = my_e;
    a.w_out[(int64_t)t * a.k + lane] = Act<TA>::from_f(my_p / psum);
    if (s_idx) s_idx[t * a.k + lane] = my_e;
  }
}

template <typename TA>
__device__ __forceinline__ void topk_dispatch(const RouterArgs<TA> &a, int t, int *s_idx) {
  if (a.E <= 128) router_topk_token<TA, 4>(a, t, s_idx);
  else if (a.E <= 256) router_topk_token<TA, 8>(a, t, s_idx);
  else if (a.E <= 512) router_topk_token<TA, 16>(a, t, s_idx);
  else router_topk_token<TA, 32>(a, t, s_idx);
}

// kTB: most tokens per token tile (1, 2, 4, 8 or 16), so the per-token
// accumulators stay in registers and no unused unrolled work executes.
template <typename TA, int kTB>
__global__ void __launch_bounds__(kRouterThreads) k1_router(RouterArgs<TA> a) {
  extern __shared__ __align__(128) uint8_t r_smem[];  // token tile (act dtype), reused by the plan
  TA *xs = reinterpret_cast<TA *>(r_smem);
  __shared__ __align__(8) uint64_t bar;
  __shared__ int s_flag;
  __shared__ int s_idx[8 * 32];  // top-k of a single-tile call (T * k <= 256), for the plan
  constexpr int V = 16 / sizeof(TA);
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int et = blockIdx.x, tt = blockIdx.y;
  const int t0 = tt * a.TB;
  const int nt = min(a.TB, a.T - t0);
  const int e_begin = et * a.EPW * kRouterWarps;
  const int e_end = min(a.E, e_begin + a.EPW * kRouterWarps);
  const int nvec = a.H / V;           // 16-byte vectors per row
  const int vpl = min(nvec / 32, kRowVecs);  // of them per lane held in registers (nvec % 32 == 0)
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrEnter);
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  // this warp's first expert row goes to registers before the dependency wait
  uint4 row[kRowVecs];
  const int e_first = e_begin + w;
  if (e_first < e_end) {
    const uint4 *src = reinterpret_cast<const uint4 *>(a.w + (int64_t)e_first * a.H);
#pragma unroll
    for (int i = 0; i < kRowVecs; ++i)
      if (i < vpl) row[i] = ldg_stream(src + i * 32 + lane);
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // x comes from the previous kernel
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrWaited);
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)nt * a.H * sizeof(TA);
    mbar_arrive_expect_tx(&bar, bytes);
    tma_bulk_g2s(xs, a.x + (int64_t)t0 * a.H, bytes, &bar);
  }
  const bool ok = mbar_wait_bounded(&bar, 0);
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      atomicOr(a.pp.status, TM_STATUS_TIMEOUT);
      mbar_wait_bounded(&bar, 0);
    }
    return;
  }
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrData);
  for (int e = e_first; e < e_end; e += kRouterWarps) {
    const bool regs = e == e_first;
    const uint4 *src = reinterpret_cast<const uint4 *>(a.w + (int64_t)e * a.H);
    float acc[kTB];
#pragma unroll
    for (int j = 0; j < kTB; ++j) acc[j] = 0.f;
#pragma unroll
    for (int i = 0; i < kRowVecs; ++i) {
      if (i < vpl) {
        const int v = i * 32 + lane;
        const uint4 q = regs ? row[i] : __ldg(src + v);
        const TA *qe = reinterpret_cast<const TA *>(&q);
        float wf[V];
#pragma unroll
        for (int u = 0; u < V; ++u) wf[u] = Act<TA>::to_f(qe[u]);
#pragma unroll
        for (int j = 0; j < kTB; ++j) {
          if (j < nt) {
            const uint4 xq = *reinterpret_cast<const uint4 *>(xs + (int64_t)j * a.H + v * V);
            const TA *xe = reinterpret_cast<const TA *>(&xq);
#pragma unroll
            for (int u = 0; u < V; ++u) acc[j] = fmaf(wf[u], Act<TA>::to_f(xe[u]), acc[j]);
          }
        }
      }
    }
    // rows longer than kRowVecs vectors per lane: the remainder, loaded in place
    for (int v = kRowVecs * 32 + lane; v < nvec; v += 32) {
      const uint4 q = __ldg(src + v);
      const TA *qe = reinterpret_cast<const TA *>(&q);
#pragma unroll
      for (int j = 0; j < kTB; ++j) {
        if (j < nt) {
          const uint4 xq = *reinterpret_cast<const uint4 *>(xs + (int64_t)j * a.H + v * V);
          const TA *xe = reinterpret_cast<const TA *>(&xq);
          for (int u = 0; u < V; ++u) acc[j] = fmaf(Act<TA>::to_f(qe[u]), Act<TA>::to_f(xe[u]), acc[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < kTB; ++j) {
      if (j < nt) {
        const float s = warp_sum(acc[j]);
        if (lane == 0) {
          const float r = Act<TA>::round(s);  // F.linear output in act dtype
          a.logits_ws[(int64_t)(t0 + j) * a.E + e] = r;
          if (a.logits_out) a.logits_out[(int64_t)(t0 + j) * a.E + e] = Act<TA>::from_f(r);
        }
      }
    }
  }
  // the last expert tile of this token tile finishes the tokens
  __threadfence();
  __syncthreads();
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrExit);
  if (tid == 0) {
    const int prev = atomicAdd(&a.tile_cnt[tt], 1);
    s_flag = (prev == a.n_etiles - 1);
    if (s_flag) a.tile_cnt[tt] = 0;
  }
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, 4);  // last CTA: top-k starts
  const bool single_tile = a.n_ttiles == 1 && a.T * a.k <= 8 * 32;
  for (int j = w; j < nt; j += kRouterWarps) topk_dispatch<TA>(a, t0 + j, single_tile ? s_idx : nullptr);
  if (!single_tile) {
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const int prev = atomicAdd(&a.tile_cnt[kMaxTokenTiles], 1);
      s_flag = (prev == a.n_ttiles - 1);
      if (s_flag) a.tile_cnt[kMaxTokenTiles] = 0;
    }
    __syncthreads();
    if (!s_flag) return;
    __threadfence();
  } else {
    __syncthreads();  // s_idx complete
  }
  const IdxSource src{a.idx_out, single_tile ? s_idx : nullptr};
  if (a.T * a.k <= 32) {
    // decode-sized call: warp 0 plans in registers while the others zero the
    // expert kernels' counters
    TM_TRACE_EVENT(a.pp.trace, kTrRouter, 5);  // plan starts
    if (w == 0) {
      plan_small_warp(src, a.T, a.k, a.E, a.pp);
      TM_TRACE_EVENT(a.pp.trace, kTrRouter, 6);  // plan done
    } else {
      for (int i = tid - 32; i < a.pp.k2_cnt_n; i += kRouterThreads - 32) a.pp.k2_cnt[i] = 0;
      for (int i = tid - 32; i < a.pp.k3_cnt_n; i += kRouterThreads - 32) a.pp.k3_cnt[i] = 0;
    }
    return;
  }
  plan_build(src, a.T, a.k, a.E, a.pp, reinterpret_cast<int *>(r_smem));
}

__global__ void __launch_bounds__(1024) k1_plan_only(const int64_t *idx, int T, int k, int E, PlanPtrs pp) {
  extern __shared__ int sm[];
  pdl_wait();
  if (T * k <= 32) {
    if (threadIdx.x < 32) {
      plan_small_warp(IdxSource{idx, nullptr}, T, k, E, pp);
    } else {
      for (int i = threadIdx.x - 32; i < pp.k2_cnt_n; i += blockDim.x - 32) pp.k2_cnt[i] = 0;
      for (int i = threadIdx.x - 32; i < pp.k3_cnt_n; i += blockDim.x - 32) pp.k3_cnt[i] = 0;
    }
    return;
  }
  plan_build(IdxSource{idx, nullptr}, T, k, E, pp, sm);
}

static size_t plan_smem(int nwarps, int E) { return sizeof(int) * ((size_t)nwarps * E + 3 * E + 64); }

// ------------------------------------------------ decode router (cluster) ----
// 16-bit logits order like their bit patterns once the sign is folded in, so a
// (logit, expert) pair packs into one u32 whose maximum is the largest logit
// with the lowest expert id: one redux.sync per top-k round.
template <typename TA> struct LogitKey;
template <> struct LogitKey<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t bits(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }
  static __device__ __forceinline__ float value(uint32_t b) { return __bfloat162float(__ushort_as_bfloat16((unsigned short)b)); }
};
template <> struct LogitKey<__half> {
  static __device__ __forceinline__ uint32_t bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
  static __device__ __forceinline__ float value(uint32_t b) { return __half2float(__ushort_as_half((unsigned short)b)); }
};
__device__ __forceinline__ uint32_t order16(uint32_t b) {
  if (b == 0x8000u) b = 0;  // -0 == +0
  return (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
}
__device__ __forceinline__ uint32_t unorder16(uint32_t k) { return (k & 0x8000u) ? (k & 0x7FFFu) : (~k & 0xFFFFu); }

// Top-k of one token from logits in shared memory (one warp); the ids also go
// to s_idx[0..k) when given (local or another CTA's shared memory).  With
// `plan` (a single-token call) the same warp also writes the routing plan.
template <typename TA, int EPL>
__device__ void topk_redux_token(const RouterArgs<TA> &a, const float *lg, int t, int *s_idx, bool plan) {
  const int lane = threadIdx.x & 31;
  float v[EPL];
  uint32_t key[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < a.E ? lg[e] : -INFINITY;
    key[i] = e < a.E ? (order16(LogitKey<TA>::bits(v[i])) << 16) | (0xFFFFu - e) : 0u;
  }
  unsigned taken = 0;
  float m = 0.f, my_v = 0.f;
  int my_e = 0;
  for (int r = 0; r < a.k; ++r) {
    uint32_t loc = 0;
#pragma unroll
    for (int i = 0; i < EPL; ++i)
      if (!(taken & (1u << i))) loc = max(loc, key[i]);
    const uint32_t win = __reduce_max_sync(0xffffffffu, loc);
    const int e = 0xFFFF - (int)(win & 0xFFFFu);
    if ((e & 31) == lane) taken |= 1u << (e >> 5);
    const float val = LogitKey<TA>::value(unorder16(win >> 16));
    if (r == 0) m = val;
    if (lane == r) { my_e = e; my_v = val; }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i)
    if (i * 32 + lane < a.E) s += __expf(v[i] - m);
  s = warp_sum(s);
  const float p = lane < a.k ? __expf(my_v - m) / s : 0.f;  // softmax probability of rank `lane`
  const float psum = warp_sum(p);
  if (lane < a.k) {
    a.idx_out[(int64_t)t * a.k + lane] = my_e;
    a.w_out[(int64_t)t * a.k + lane] = Act<TA>::from_f(p / psum);
    if (s_idx) s_idx[lane] = my_e;
  }
  if (!plan) return;
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, 5);  // top-k done, plan starts
  // single token: the k distinct experts each get one slot, in ascending id order
  int asc = 0;
  for (int q = 0; q < a.k; ++q) asc += __shfl_sync(0xffffffffu, my_e, q) < my_e;
  const PlanPtrs &pp = a.pp;
  if (lane < a.k) {
    pp.slot_pair[asc] = lane;
    pp.slot_token[asc] = 0;
    pp.pair_slot[lane] = asc;
    pp.act_list[asc] = my_e;
    pp.act_rec[asc] = make_int4(my_e, 1, asc, 0);
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int x = i * 32 + lane;
    int below = 0;
    for (int q = 0; q < a.k; ++q) below += __shfl_sync(0xffffffffu, my_e, q) < x;
    if (x < a.E) {
      pp.counts[x] = (taken >> i) & 1u;
      pp.offsets[x] = below;
    }
  }
  if (lane == 0) {
    pp.offsets[a.E] = a.k;
    pp.meta[kMetaNActive] = a.k;
    pp.meta[kMetaPairs] = a.k;
    pp.meta[kMetaTokens] = 1;
  }
}

// Decode router: one cluster of kClusterCTAs CTAs, two expert rows per warp
// (held in registers before the dependency wait).  Every CTA writes its
// logits straight into CTA 0's shared memory; after the cluster barrier CTA 0
// selects the top-k and writes the plan.  No global atomics or fences.
template <typename TA, int kTB>
__global__ void __launch_bounds__(kRouterThreads) k1_router_cluster(RouterArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  extern __shared__ __align__(128) uint8_t r_smem[];  // token tile, then (CTA 0) the plan's scratch
  TA *xs = reinterpret_cast<TA *>(r_smem);
  __shared__ float s_logit[kClusterMaxT][kClusterMaxE];
  __shared__ int s_idx[kClusterMaxT * 32];
  __shared__ __align__(8) uint64_t bar;
  constexpr int V = 8;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nt = a.T;
  const int nvec = a.H / V, vpl = nvec / 32;  // <= 8 (host checks)
  const int e0 = crank * (kRouterWarps * 2) + w * 2;
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrEnter);
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  uint4 row[2][8];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    if (e0 + r < a.E) {
      const uint4 *src = reinterpret_cast<const uint4 *>(a.w + (int64_t)(e0 + r) * a.H);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < vpl) row[r][i] = ldg_stream(src + i * 32 + lane);
    }
  }
  __syncthreads();
  pdl_trigger();
  pdl_wait();  // x comes from the previous kernel
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrWaited);
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)nt * a.H * sizeof(TA);
    mbar_arrive_expect_tx(&bar, bytes);
    tma_bulk_g2s(xs, a.x, bytes, &bar);
  }
  const bool ok = !__syncthreads_or(!mbar_wait_bounded(&bar, 0));
  if (!ok && tid == 0) {
    atomicOr(a.pp.status, TM_STATUS_TIMEOUT);
    mbar_wait_bounded(&bar, 0);
  }
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrData);
  float *logit0 = cluster.map_shared_rank(&s_logit[0][0], 0);
  if (ok) {
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int e = e0 + r;
      if (e >= a.E) continue;
      float acc[kTB];
#pragma unroll
      for (int j = 0; j < kTB; ++j) acc[j] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (i < vpl) {
          const int vv = i * 32 + lane;
          const TA *qe = reinterpret_cast<const TA *>(&row[r][i]);
          float wf[V];
#pragma unroll
          for (int u = 0; u < V; ++u) wf[u] = Act<TA>::to_f(qe[u]);
#pragma unroll
          for (int j = 0; j < kTB; ++j) {
            if (j < nt) {
              const uint4 xq = *reinterpret_cast<const uint4 *>(xs + (int64_t)j * a.H + vv * V);
              const TA *xe = reinterpret_cast<const TA *>(&xq);
#pragma unroll
              for (int u = 0; u < V; ++u) acc[j] = fmaf(wf[u], Act<TA>::to_f(xe[u]), acc[j]);
            }
          }
        }
      }
#pragma unroll
      for (int j = 0; j < kTB; ++j) {
        if (j < nt) {
          const float s = warp_sum(acc[j]);
          if (lane == 0) {
            const float rr = Act<TA>::round(s);  // F.linear output in act dtype
            logit0[j * kClusterMaxE + e] = rr;
            if (a.logits_out) a.logits_out[(int64_t)j * a.E + e] = Act<TA>::from_f(rr);
          }
        }
      }
    }
  }
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, 4);  // dot products done
  cluster.sync();  // every CTA's logits are in CTA 0
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrExit);
  if (crank != 0 || !ok) return;
  if (nt == 1) {
    if (w == 0) {
      topk_redux_token<TA, kClusterMaxE / 32>(a, s_logit[0], 0, nullptr, true);
      TM_TRACE_EVENT(a.pp.trace, kTrRouter, 6);
    } else {
      for (int i = tid - 32; i < a.pp.k3_cnt_n; i += kRouterThreads - 32) a.pp.k3_cnt[i] = 0;
    }
    return;
  }
  if (w < nt) topk_redux_token<TA, kClusterMaxE / 32>(a, s_logit[w], w, s_idx + w * a.k, false);
  __syncthreads();
  const IdxSource src{a.idx_out, s_idx};
  if (nt * a.k <= 32) {
    if (w == 0) {
      plan_small_warp(src, nt, a.k, a.E, a.pp);
    } else {
      for (int i = tid - 32; i < a.pp.k3_cnt_n; i += kRouterThreads - 32) a.pp.k3_cnt[i] = 0;
    }
    return;
  }
  plan_build(src, nt, a.k, a.E, a.pp, reinterpret_cast<int *>(r_smem));
}

// One-token decode router (k <= 8, E <= 128): the latency-critical link of
// every decode layer, so each stage is a short dependency chain.
//  * One expert row per warp (16 warps per CTA, 8 CTAs), held in registers
//    before the dependency wait; the dot product runs as 4 independent
//    partial sums.
//  * Each warp sends its logit into CTA 0's shared memory with st.async,
//    which completes 4 bytes on CTA 0's mbarrier (CTA 0 expects 4 * E): no
//    fence, no cluster-wide barrier; only CTA 0's warp 0 waits.
//  * Top-k: each lane sorts its 4 (logit, expert) keys, then k rounds of one
//    redux.sync.max over the lanes' heads, the winner advancing; the softmax
//    denominator's reduction runs between those rounds.
//  * The plan comes from a 128-bit mask of the selected experts (popcounts),
//    not from shuffles.
// Same results as k1_router_cluster: the same keys and tie rule (value
// descending, then lower expert id), the same softmax and renormalisation
// arithmetic in the same order; the logits' fp32 partial sums are added in a
// different order (within the rounding the tests allow for F.linear).
constexpr int kT1MaxK = 8;
constexpr int kT1Warps = kClusterMaxE / kClusterCTAs;  // 16: one expert row per warp
constexpr int kT1Threads = kT1Warps * 32;
template <typename TA, bool kNorm>
__global__ void __launch_bounds__(kT1Threads) k1_router_t1(RouterArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  extern __shared__ __align__(128) uint8_t r_smem[];  // x row
  TA *xs = reinterpret_cast<TA *>(r_smem);
  __shared__ __align__(16) float s_logit[kClusterMaxE];
  __shared__ __align__(8) uint64_t bar;   // x copy
  __shared__ __align__(8) uint64_t lbar;  // CTA 0: 4 * E bytes of logits from the cluster
  __shared__ float nred[8];
  constexpr int V = 8;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int vpl = a.H / (V * 32);  // 16-byte vectors per lane (<= 8: host checks)
  const int e = crank * kT1Warps + w;
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrEnter);
  if (tid == 0) {
    mbar_init(&bar, 1);
    mbar_init(&lbar, 1);
    mbar_init_fence_cluster();
    if (crank == 0) mbar_arrive_expect_tx(&lbar, (uint32_t)a.E * 4u);
  }
  uint4 row[8];
  {
    const uint4 *src = reinterpret_cast<const uint4 *>(a.w + (int64_t)min(e, a.E - 1) * a.H);
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < vpl) row[i] = ldg_stream(src + i * 32 + lane);
  }
  // RMSNorm weights (independent of the previous kernel): threads 0-255 own
  // elements (c * 256 + tid) * 4 .. + 3, c < 4, as k8_rmsnorm does
  constexpr bool norm = kNorm;   // a separate instance: the plain router keeps its registers
  float nwv[4][4];
#pragma unroll
  for (int c = 0; c < 4; ++c)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = (c * 256 + tid) * 4 + e;
      nwv[c][e] = (norm && tid < 256 && i < a.H) ? Act<TA>::to_f(a.norm_w[i]) : 0.f;
    }
  cluster.sync();  // every CTA runs and CTA 0's lbar is initialised (off the critical path)
  pdl_trigger();
  pdl_wait();  // x comes from the previous kernel
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrWaited);
  if (tid == 0) {
    const uint32_t bytes = (uint32_t)a.H * sizeof(TA);
    mbar_arrive_expect_tx(&bar, bytes);
    tma_bulk_g2s(xs, a.x, bytes, &bar);
  }
  const bool ok = mbar_wait_bounded(&bar, 0);
  if (!ok && lane == 0) atomicOr(a.pp.status, TM_STATUS_TIMEOUT);
  if (norm) {
    // Qwen3MoeRMSNorm of the token on threads 0-255 with k8_rmsnorm's sums in
    // its order (the same bits in every CTA of the cluster and as the
    // separate kernel); the normalised token replaces x in shared memory
    float v[4][4];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int i = (c * 256 + tid) * 4;
#pragma unroll
      for (int e = 0; e < 4; ++e) v[c][e] = 0.f;
      if (tid < 256 && i < a.H) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v[c][e] = Act<TA>::to_f(xs[i + e]);
          ss = fmaf(v[c][e], v[c][e], ss);
        }
      }
    }
    ss = warp_sum(ss);
    if (lane == 0 && w < 8) nred[w] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += nred[i];
    const float r = rsqrtf(tot / (float)a.H + a.eps);
    if (tid < 256) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int i = (c * 256 + tid) * 4;
        if (i < a.H) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const TA y = Act<TA>::from_f(Act<TA>::round(v[c][e] * r) * nwv[c][e]);
            xs[i + e] = y;
            if (crank == 0) a.x_norm_out[i + e] = y;
          }
        }
      }
    }
    __syncthreads();
  }
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrData);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < vpl) {
      const uint4 xq = *reinterpret_cast<const uint4 *>(xs + (i * 32 + lane) * V);
      const TA *xe = reinterpret_cast<const TA *>(&xq);
      const TA *qe = reinterpret_cast<const TA *>(&row[i]);
#pragma unroll
      for (int u = 0; u < V; ++u) acc[u & 3] = fmaf(Act<TA>::to_f(qe[u]), Act<TA>::to_f(xe[u]), acc[u & 3]);
    }
  }
  float sum = (acc[0] + acc[1]) + (acc[2] + acc[3]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, 7);  // dot product reduced
  if (lane == 0 && e < a.E) {
    const float r = Act<TA>::round(sum);  // F.linear output in act dtype
    st_async_u32(cluster_addr(&s_logit[e], 0), __float_as_uint(r), cluster_addr(&lbar, 0));
    if (a.logits_out) a.logits_out[e] = Act<TA>::from_f(r);
  }
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, 4);  // logit sent
  if (crank != 0) return;
  if (w != 0) {
    for (int i = tid - 32; i < a.pp.k3_cnt_n; i += kT1Threads - 32) a.pp.k3_cnt[i] = 0;
    return;
  }
  // CTA 0, warp 0.  Its limit is above every peer's own x wait (1 s), so a
  // peer always has sent its logit before this gives up.
  if (!mbar_wait_cluster_bounded(&lbar, 0, 2000000000ull)) {
    if (lane == 0) atomicOr(a.pp.status, TM_STATUS_TIMEOUT);
    return;
  }
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrExit);
  // ---- top-k over 4 keys per lane (expert i * 32 + lane)
  float v[4];
  uint32_t key[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int e = i * 32 + lane;
    v[i] = e < a.E ? s_logit[e] : -INFINITY;
    key[i] = e < a.E ? (order16(LogitKey<TA>::bits(v[i])) << 16) | (0xFFFFu - e) : 0u;
  }
  uint32_t h0 = max(key[0], key[1]), h1 = min(key[0], key[1]);  // sort descending
  uint32_t h2 = max(key[2], key[3]), h3 = min(key[2], key[3]);
  {
    const uint32_t a0 = max(h0, h2), a2 = min(h0, h2), a1 = max(h1, h3), a3 = min(h1, h3);
    h0 = a0;
    h1 = max(a1, a2);
    h2 = min(a1, a2);
    h3 = a3;
  }
  uint32_t win[kT1MaxK];
  float m = 0.f, ls = 0.f;
#pragma unroll
  for (int r = 0; r < kT1MaxK; ++r) {
    if (r < a.k) {
      win[r] = __reduce_max_sync(0xffffffffu, h0);
      if (h0 == win[r]) {  // keys are distinct: exactly one lane advances
        h0 = h1;
        h1 = h2;
        h2 = h3;
        h3 = 0u;
      }
    } else {
      win[r] = 0u;
    }
    if (r == 0) {  // softmax denominator: exp(v - max) summed in expert-slot order, then over lanes
      m = LogitKey<TA>::value(unorder16(win[0] >> 16));
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (i * 32 + lane < a.E) ls += __expf(v[i] - m);
    } else if (r <= 5) {
      ls += __shfl_xor_sync(0xffffffffu, ls, 32 >> r);
    }
  }
  // rank `lane` (< k): its expert and logit
  int my_e = 0;
  float my_v = 0.f;
#pragma unroll
  for (int r = 0; r < kT1MaxK; ++r)
    if (lane == r) {
      my_e = 0xFFFF - (int)(win[r] & 0xFFFFu);
      my_v = LogitKey<TA>::value(unorder16(win[r] >> 16));
    }
  const float p = lane < a.k ? __expf(my_v - m) / ls : 0.f;  // softmax probability of rank `lane`
  const float psum = warp_sum(p);
  // ---- plan: mask of the selected experts
  uint32_t msk[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int r = 0; r < kT1MaxK; ++r) {
    if (r < a.k) {
      const int e = 0xFFFF - (int)(win[r] & 0xFFFFu);
#pragma unroll
      for (int i = 0; i < 4; ++i) msk[i] |= (e >> 5) == i ? 1u << (e & 31) : 0u;
    }
  }
  const PlanPtrs &pp = a.pp;
  int below = 0;  // selected experts with an id below i * 32 + lane
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int x = i * 32 + lane;
    const int here = below + __popc(msk[i] & ((1u << lane) - 1u));
    if (x < a.E) {
      pp.counts[x] = (msk[i] >> lane) & 1u;
      pp.offsets[x] = here;
    }
    below += __popc(msk[i]);
  }
  if (lane < a.k) {
    const int ew = my_e >> 5, eb = my_e & 31;
    int asc = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i)  // (selects, not a dynamically indexed register array)
      asc += i < ew ? __popc(msk[i]) : i == ew ? __popc(msk[i] & ((1u << eb) - 1u)) : 0;
    a.idx_out[lane] = my_e;
    a.w_out[lane] = Act<TA>::from_f(p / psum);
    pp.slot_pair[asc] = lane;
    pp.slot_token[asc] = 0;
    pp.pair_slot[lane] = asc;
    pp.act_list[asc] = my_e;
    pp.act_rec[asc] = make_int4(my_e, 1, asc, 0);
  }
  if (lane == 0) {
    pp.offsets[a.E] = a.k;
    pp.meta[kMetaNActive] = a.k;
    pp.meta[kMetaPairs] = a.k;
    pp.meta[kMetaTokens] = 1;
  }
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, 6);
}

// ------------------------------------- multi-token router (tensor cores) ----
// Every 16-bit call the decode router does not take: one thread-block cluster
// of kClusterCTAs CTAs per tile of kTcTile tokens.  CTA r of a cluster takes
// the r-th eighth of the hidden dimension (in 32-element chunks) for every
// expert; warp w covers experts [w*8*NT, (w+1)*8*NT) on mma.sync m16n8k16
// (16-bit operands, fp32 accumulators).  The order of the reduction dimension
// inside one MMA is free as long as A and B use the same one, so every lane
// loads 16 contiguous bytes of its token rows and of its expert row and feeds
// them to two MMAs (no shared-memory staging).  The eight partial sums of a
// token go to the CTA that owns it (token j of a tile: CTA j % 8), which adds
// them in CTA order, rounds to the act dtype (F.linear's output) and selects
// the top-k.  A one-tile call also builds the routing plan in CTA 0; larger
// calls leave it to k1_plan_scatter.
constexpr int kTcTile = 16;

template <typename TA> struct MmaAct;
template <> struct MmaAct<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    mma_16816(d, a0, a1, a2, a3, b0, b1);
  }
};
template <> struct MmaAct<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
  }
};

template <typename TA>
__device__ __forceinline__ void topk_redux_dispatch(const RouterArgs<TA> &a, const float *lg, int t, int *s_idx) {
  if (a.E <= 128) topk_redux_token<TA, 4>(a, lg, t, s_idx, false);
  else if (a.E <= 256) topk_redux_token<TA, 8>(a, lg, t, s_idx, false);
  else if (a.E <= 512) topk_redux_token<TA, 16>(a, lg, t, s_idx, false);
  else topk_redux_token<TA, 32>(a, lg, t, s_idx, false);
}

constexpr int kTcMaxMT = 4;  // m16 tiles per cluster (64 tokens)
constexpr int kTcPass = 8;   // 32-element chunks of the token tile staged in shared memory per pass
constexpr int kTcRowB = kTcPass * 64;  // bytes of one staged token row

// Chunks of router weights a lane keeps in flight (NT 16-byte vectors each).
template <int NT, int MT> struct TcDepth {
  static constexpr int value = NT <= 2 ? 4 : (NT <= 4 && MT == 1) ? 2 : 1;  // no spills at 128 registers
};

// MT m16 tiles (16 * MT tokens) per cluster; token j of a tile belongs to CTA
// j % 8 as its row j / 8.  The CTA's slice of the token tile is staged once
// in shared memory by cp.async (16-byte units, odd rows XOR-swizzled by 64
// bytes so that the eight rows a warp reads per step fall on distinct banks)
// and read by all eight warps; each warp's router rows stream from L2 into
// registers, TcDepth chunks ahead (the first before griddepcontrol.wait).
// Every accumulator sees the same MMA sequence as a lane loading its 16-byte
// token and router vectors straight from global memory: chunks ascending, two
// MMAs per chunk over the same element pairs.  64-token tiles are held to 128
// registers (two CTAs per SM).  Dynamic shared memory: partial logits
// [kClusterCTAs][2 * MT][Ec] (Ec = 64 * NT experts; later the plan's scratch
// in CTA 0 of a one-tile call), then the staged token rows [16 * MT][kTcRowB].
template <typename TA, int NT, int MT>
__global__ void __launch_bounds__(kRouterThreads, MT == 4 ? 2 : 1) k1_router_tc(RouterArgs<TA> a) {
  static_assert(sizeof(TA) == 2, "16-bit activations");
  static_assert(2 * MT <= kRouterWarps, "one warp per owned token");
  extern __shared__ __align__(16) float tc_part[];
  __shared__ int s_tidx[kTcTile * kTcMaxMT * 32];  // CTA 0: the tile's top-k ids
  constexpr int EW = 8 * NT;                 // experts per warp
  constexpr int Ec = kRouterWarps * EW;      // experts per CTA (>= E)
  constexpr int R = 2 * MT;                  // rows (tokens) owned per CTA
  constexpr int WD = TcDepth<NT, MT>::value;     // router-weight chunks in flight
  static_assert(kTcPass % WD == 0 && kTcPass / 2 % WD == 0, "passes split into whole groups");
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = (int)cluster.block_rank();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g = lane >> 2, c = lane & 3;
  const int t0 = blockIdx.y * (kTcTile * MT);
  const int nt = min(kTcTile * MT, a.T - t0);
  const int nchunk = a.H / 32;
  const int c_lo = crank * nchunk / kClusterCTAs, c_hi = (crank + 1) * nchunk / kClusterCTAs;
  char *xs = reinterpret_cast<char *>(tc_part + kClusterCTAs * R * Ec);
  const uint32_t xs_u32 = smem_u32(xs);
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrEnter);
  // every CTA of the cluster has started before any writes into another's shared memory
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  // this CTA's slice of the router weights does not depend on the previous kernel
  {
    const int row_bytes = (c_hi - c_lo) * 64;  // 32 elements x 2 bytes per chunk
    const int lines = (row_bytes + 127) / 128;
    for (int i = tid; i < a.E * lines; i += kRouterThreads) {
      const int e = i / lines, l = i - e * lines;
      const char *p = reinterpret_cast<const char *>(a.w + (int64_t)e * a.H + c_lo * 32) + l * 128;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
    }
  }
  const uint4 *wr[NT];
  bool we[NT];
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    const int e = w * EW + 8 * j + g;
    we[j] = e < a.E;
    wr[j] = reinterpret_cast<const uint4 *>(a.w + (int64_t)(we[j] ? e : 0) * a.H) + c;
  }
  const uint4 z = make_uint4(0u, 0u, 0u, 0u);
  uint4 wq[WD][NT];  // chunk c_lo + i * WD + u sits in wq[u]
#pragma unroll
  for (int u = 0; u < WD; ++u)
#pragma unroll
    for (int j = 0; j < NT; ++j) wq[u][j] = (c_lo + u < c_hi && we[j]) ? __ldg(wr[j] + (c_lo + u) * 4) : z;
  pdl_trigger();
  pdl_wait();  // x comes from the previous kernel
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrWaited);
  float acc[MT][NT][4];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < NT; ++j) acc[m][j][0] = acc[m][j][1] = acc[m][j][2] = acc[m][j][3] = 0.f;
  const uint32_t swz = (uint32_t)(g & 1) << 2;  // rows 16m + 8h + g share g's parity
  for (int p0 = c_lo; p0 < c_hi; p0 += kTcPass) {
    const int npc = min(kTcPass, c_hi - p0);
    if (p0 != c_lo) __syncthreads();  // every warp is done with the previous pass
    // stage the pass: rows [0, 16 * MT) (zero past the call's tokens), two groups of chunks
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int qa = half * (kTcPass / 2), qb = min(npc, qa + kTcPass / 2);
      const int per_row = max(0, qb - qa) * 4;  // 16-byte units
      for (int i = tid; i < kTcTile * MT * per_row; i += kRouterThreads) {
        const int r = i / per_row, u = qa * 4 + (i - r * per_row);
        const bool in = r < nt;
        const TA *src = a.x + (int64_t)(t0 + (in ? r : 0)) * a.H + (p0 + (u >> 2)) * 32 + (u & 3) * 8;
        cp_async16_z(xs_u32 + r * kTcRowB + ((u ^ ((r & 1) << 2)) << 4), src, in ? 16 : 0);
      }
      cp_async_commit();
    }
#pragma unroll
    for (int b = 0; b < kTcPass; b += WD) {
      if (b >= npc) break;  // uniform over the CTA
      if (b == 0) {
        cp_async_wait<1>();
        __syncthreads();
      } else if (b == kTcPass / 2) {
        cp_async_wait<0>();
        __syncthreads();
      }
#pragma unroll
      for (int u = 0; u < WD; ++u) {
        const int q = b + u;
        if (q < npc) {
          const uint32_t col = ((uint32_t)(q * 4 + c) ^ swz) << 4;
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const uint4 p = *reinterpret_cast<const uint4 *>(xs + (16 * m + g) * kTcRowB + col);
            const uint4 qv = *reinterpret_cast<const uint4 *>(xs + (16 * m + 8 + g) * kTcRowB + col);
#pragma unroll
            for (int j = 0; j < NT; ++j) {
              const uint4 &bv = wq[u][j];
              MmaAct<TA>::run(acc[m][j], p.x, qv.x, p.y, qv.y, bv.x, bv.y);
              MmaAct<TA>::run(acc[m][j], p.z, qv.z, p.w, qv.w, bv.z, bv.w);
            }
          }
          const int nch = p0 + q + WD;
#pragma unroll
          for (int j = 0; j < NT; ++j) wq[u][j] = (nch < c_hi && we[j]) ? __ldg(wr[j] + nch * 4) : z;
        }
      }
    }
  }
  asm volatile("barrier.cluster.wait.aligned;" ::: "memory");
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrData);
  // rows 16m + g and 16m + g + 8 belong to CTA g as its rows 2m and 2m + 1
  float *dst = cluster.map_shared_rank(tc_part, g);
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const int e = w * EW + 8 * j + 2 * c;
      *reinterpret_cast<float2 *>(dst + (crank * R + 2 * m) * Ec + e) = make_float2(acc[m][j][0], acc[m][j][1]);
      *reinterpret_cast<float2 *>(dst + (crank * R + 2 * m + 1) * Ec + e) = make_float2(acc[m][j][2], acc[m][j][3]);
    }
  cluster.sync();  // every partial of this CTA's tokens has arrived
  for (int i = tid; i < R * a.E; i += kRouterThreads) {
    const int r = i / a.E, e = i - r * a.E;
    float s = 0.f;
#pragma unroll
    for (int src = 0; src < kClusterCTAs; ++src) s += tc_part[(src * R + r) * Ec + e];
    const float v = Act<TA>::round(s);  // F.linear output in act dtype
    tc_part[r * Ec + e] = v;            // over source 0's partial, read above by this thread only
    const int j = 8 * r + crank;        // token within the tile
    if (a.logits_out && j < nt) a.logits_out[(int64_t)(t0 + j) * a.E + e] = Act<TA>::from_f(v);
  }
  __syncthreads();
  if (w < R && 8 * w + crank < nt) {
    const int j = 8 * w + crank;
    int *tidx0 = cluster.map_shared_rank(s_tidx, 0);
    topk_redux_dispatch<TA>(a, tc_part + w * Ec, t0 + j, tidx0 + j * a.k);
  }
  TM_TRACE_EVENT(a.pp.trace, kTrRouter, kTrExit);
  cluster.sync();  // CTA 0 holds the tile's top-k ids
  if (crank != 0) return;
  if (a.n_ttiles != 1) {
    // routed pairs per expert of each 16-token unit, for k1_plan_scatter
    int *h = reinterpret_cast<int *>(tc_part);  // [MT][E]
    for (int e = tid; e < MT * a.E; e += kRouterThreads) h[e] = 0;
    __syncthreads();
    for (int p = tid; p < nt * a.k; p += kRouterThreads) {
      const int unit = p / (kTcTile * a.k);
      atomicAdd(&h[unit * a.E + s_tidx[p]], 1);  // top-k ids are < E
    }
    __syncthreads();
    const int units = (nt + kTcTile - 1) / kTcTile;
    int *dst_h = a.pp.unit_hist + (int64_t)(t0 / kTcTile) * a.E;
    for (int e = tid; e < units * a.E; e += kRouterThreads) dst_h[e] = h[e];
    return;
  }
  // one tile: CTA 0 builds the plan
  const IdxSource src{a.idx_out, s_tidx};
  if (nt * a.k <= 32) {
    if (w == 0) {
      plan_small_warp(src, nt, a.k, a.E, a.pp);
    } else {
      for (int i = tid - 32; i < a.pp.k2_cnt_n; i += kRouterThreads - 32) a.pp.k2_cnt[i] = 0;
      for (int i = tid - 32; i < a.pp.k3_cnt_n; i += kRouterThreads - 32) a.pp.k3_cnt[i] = 0;
    }
    return;
  }
  plan_build(src, nt, a.k, a.E, a.pp, reinterpret_cast<int *>(tc_part));
}

template <int NT, int MT> static size_t router_tc_smem(int E) {
  const size_t part = (size_t)kClusterCTAs * 2 * MT * kRouterWarps * 8 * NT * sizeof(float);
  // the plan's scratch (CTA 0, after the last cluster barrier) may run over the dead token rows
  return std::max(part + (size_t)kTcTile * MT * kTcRowB,
                  std::max(plan_smem(kRouterWarps, E), (size_t)MT * E * sizeof(int)));
}

// Routing plan of a call with many (token, rank) pairs, on many CTAs, from
// the per-expert counts of every 16-token unit (unit_hist).  CTA b takes units
// [b * U, (b + 1) * U): it adds up the counts of all units (totals) and of
// the units before its own, derives the expert offsets, and places its pairs:
// slot = offset[e] + earlier pairs of e, i.e. experts ascending and pair index
// ascending within an expert (the order of plan_build).  CTA 0 also writes the
// per-expert tables and zeroes the expert kernels' counters.
constexpr int kUnitTokens = 16;
static_assert(kUnitTokens == kTcTile, "k1_router_tc writes one unit_hist row per token tile");
constexpr int kScatterThreads = 512;
constexpr int kScatterWarps = kScatterThreads / 32;

static size_t plan_scatter_smem(int E) { return sizeof(int) * ((size_t)(4 + 2 * kScatterWarps) * E + 96); }

__global__ void __launch_bounds__(kScatterThreads) k1_plan_scatter(const int64_t *idx, int T, int k, int E,
                                                                   int U, PlanPtrs pp) {
  extern __shared__ int sc_sm[];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int P = T * k;
  const int n_units = (T + kUnitTokens - 1) / kUnitTokens;
  const int u_lo = blockIdx.x * U;
  const int lo = u_lo * kUnitTokens * k, hi = min(P, (u_lo + U) * kUnitTokens * k);
  int *before = sc_sm;              // [E] valid pairs of e in units before u_lo
  int *cnt = before + E;            // [E] valid pairs of e, then offsets
  int *flag = cnt + E;              // [E] active flag, then active index
  int *cnt0 = flag + E;             // [E] counts (kept)
  int *hist = cnt0 + E;             // [kScatterWarps][E]
  int *tmp = hist + kScatterWarps * E;  // [66]
  int *part_t = tmp + 96;           // [kScatterWarps][E] partial totals of the column sums
  TM_TRACE_EVENT(pp.trace, kTrPlan, kTrEnter);
  for (int i = tid; i < 2 * E; i += kScatterThreads) sc_sm[i] = 0;
  for (int i = tid; i < kScatterWarps * E; i += kScatterThreads) hist[i] = 0;
  pdl_trigger();
  pdl_wait();  // indices and unit counts come from the previous kernel
  TM_TRACE_EVENT(pp.trace, kTrPlan, kTrWaited);
  if (blockIdx.x == 0) {
    for (int i = tid; i < pp.k2_cnt_n; i += kScatterThreads) pp.k2_cnt[i] = 0;
    for (int i = tid; i < pp.k3_cnt_n; i += kScatterThreads) pp.k3_cnt[i] = 0;
  }
  __syncthreads();
  // column sums of unit_hist: q <= 16 threads per group of 4 experts (16-byte
  // loads, each over a strided set of units) leave their partials in the
  // (still unused) per-warp histogram rows and in part_t, added up per expert
  // below; or q threads per expert with shared-memory atomics when E % 4 != 0
  const bool by4 = (E & 3) == 0;
  const int q4 = by4 ? min(kScatterWarps, max(1, kScatterThreads / (E >> 2))) : 0;
  if (by4) {
    const int E4 = E >> 2;
    for (int col = tid; col < q4 * E4; col += kScatterThreads) {
      const int e4 = col % E4, part = col / E4;
      int4 sb = make_int4(0, 0, 0, 0), st = make_int4(0, 0, 0, 0);
#pragma unroll 8
      for (int u = part; u < n_units; u += q4) {
        const int4 v = __ldcg(reinterpret_cast<const int4 *>(pp.unit_hist + (int64_t)u * E) + e4);
        st.x += v.x; st.y += v.y; st.z += v.z; st.w += v.w;
        if (u < u_lo) { sb.x += v.x; sb.y += v.y; sb.z += v.z; sb.w += v.w; }
      }
      reinterpret_cast<int4 *>(hist + part * E)[e4] = sb;
      reinterpret_cast<int4 *>(part_t + part * E)[e4] = st;
    }
    __syncthreads();
    for (int x = tid; x < E; x += kScatterThreads) {
      int sb = 0, st = 0;
      for (int part = 0; part < q4; ++part) {
        sb += hist[part * E + x];
        st += part_t[part * E + x];
      }
      before[x] = sb;
      cnt[x] = st;
    }
  } else {
    const int q = max(1, kScatterThreads / E);
    for (int col = tid; col < q * E; col += kScatterThreads) {
      const int e = col % E, part = col / E;
      int sb = 0, st = 0;
#pragma unroll 8
      for (int u = part; u < n_units; u += q) {
        const int v = __ldcg(pp.unit_hist + (int64_t)u * E + e);
        st += v;
        sb += u < u_lo ? v : 0;
      }
      atomicAdd(&before[e], sb);
      atomicAdd(&cnt[e], st);
    }
  }
  __syncthreads();
  for (int x = tid; x < E; x += kScatterThreads) {
    cnt0[x] = cnt[x];
    flag[x] = cnt[x] > 0 ? 1 : 0;
  }
  __syncthreads();
  TM_TRACE_EVENT(pp.trace, kTrPlan, kTrData);  // counts of every unit added up
  const int2 tots = block_excl_scan2(cnt, flag, E, tmp);
  const int total = tots.x, n_active = tots.y;
  if (by4) {  // the partials are read (barrier inside the scan): clear the histogram rows again
    for (int i = tid; i < q4 * E; i += kScatterThreads) hist[i] = 0;  // rows written above
    __syncthreads();
  }
  TM_TRACE_EVENT(pp.trace, kTrPlan, 4);  // offsets known
  if (blockIdx.x == 0) {
    for (int x = tid; x < E; x += kScatterThreads) {
      const int c0 = cnt0[x];
      pp.counts[x] = c0;
      pp.offsets[x] = cnt[x];
      if (c0 > 0) {
        pp.act_list[flag[x]] = x;
        pp.act_rec[flag[x]] = make_int4(x, c0, cnt[x], 0);
      }
    }
    if (tid == 0) {
      pp.offsets[E] = total;
      pp.meta[kMetaNActive] = n_active;
      pp.meta[kMetaPairs] = P;
      pp.meta[kMetaTokens] = T;
    }
  }
  // this CTA's pairs: per-warp histograms, then a stable scatter (as plan_build)
  const int n = max(0, hi - lo);
  const int wlo = lo + (int)((int64_t)w * n / kScatterWarps), whi = lo + (int)((int64_t)(w + 1) * n / kScatterWarps);
  // the first kKeep groups of 32 ids stay in registers for the second pass
  constexpr int kKeep = 4;
  auto load_e = [&](int p) -> int {
    if (p >= whi) return -2;
    const int64_t v = __ldcg(idx + p);
    return (v >= 0 && v < E) ? (int)v : -1;
  };
  int keep[kKeep];
#pragma unroll
  for (int it = 0; it < kKeep; ++it) keep[it] = load_e(wlo + it * 32 + lane);
#pragma unroll
  for (int it = 0; it < kKeep; ++it)
    if (keep[it] >= 0) atomicAdd(&hist[w * E + keep[it]], 1);
  for (int b = wlo + kKeep * 32; b < whi; b += 32) {
    const int e = load_e(b + lane);
    if (e >= 0) atomicAdd(&hist[w * E + e], 1);
  }
  __syncthreads();
  TM_TRACE_EVENT(pp.trace, kTrPlan, 6);  // this CTA's per-warp histograms
  for (int x = tid; x < E; x += kScatterThreads) {
    int run = cnt[x] + before[x];
    for (int j = 0; j < kScatterWarps; ++j) {
      const int c0 = hist[j * E + x];
      hist[j * E + x] = run;
      run += c0;
    }
  }
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  auto place = [&](int p, int e) {
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt_mask);
    if (e >= 0) {
      const int slot = hist[w * E + e] + rank;
      pp.slot_pair[slot] = p;
      pp.slot_token[slot] = p / k;
      pp.pair_slot[p] = slot;
    } else if (e == -1) {
      pp.pair_slot[p] = -1;
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) hist[w * E + e] += __popc(peers);
    __syncwarp();
  };
#pragma unroll
  for (int it = 0; it < kKeep; ++it)
    if (wlo + it * 32 < whi) place(wlo + it * 32 + lane, keep[it]);
  for (int b = wlo + kKeep * 32; b < whi; b += 32) place(b + lane, load_e(b + lane));
  TM_TRACE_EVENT(pp.trace, kTrPlan, kTrExit);
}

// unit_hist from top-k indices given by the caller: one CTA per 16-token unit.
__global__ void __launch_bounds__(256) k1_plan_hist(const int64_t *idx, int T, int k, int E, PlanPtrs pp) {
  extern __shared__ int ph_sm[];
  const int tid = threadIdx.x;
  const int t0 = blockIdx.x * kUnitTokens, nt = min(kUnitTokens, T - t0);
  for (int e = tid; e < E; e += blockDim.x) ph_sm[e] = 0;
  pdl_trigger();
  pdl_wait();
  __syncthreads();
  bool bad = false;
  for (int p = tid; p < nt * k; p += blockDim.x) {
    const int64_t v = __ldcg(idx + (int64_t)t0 * k + p);
    if (v >= 0 && v < E) atomicAdd(&ph_sm[(int)v], 1);
    else bad = true;
  }
  if (__any_sync(0xffffffffu, bad) && (tid & 31) == 0) atomicOr(pp.status, TM_STATUS_BAD_EXPERT_ID);
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) pp.unit_hist[(int64_t)blockIdx.x * E + e] = ph_sm[e];
}

// CTAs and units per CTA of k1_plan_scatter for T tokens.
static void plan_scatter_grid(int64_t T, int *ctas, int *units) {
  const int64_t n_units = (T + kUnitTokens - 1) / kUnitTokens;
  const int64_t n = std::min<int64_t>(n_units, 148);
  *units = (int)((n_units + n - 1) / n);
  *ctas = (int)((n_units + *units - 1) / *units);
}
template <typename Kern, typename... Args>
static int launch_cluster_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, int cluster_x, cudaStream_t s,
                              const char *what, Args... args) {
  int rc = ensure_smem(reinterpret_cast<const void *>(kernel), smem);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  return cuda_check(cudaLaunchKernelEx(&cfg, kernel, args...), what);
}


struct RouterLaunch {
  const void *x, *w;
  int64_t *idx;
  void *wout, *logits;
  void *ws;
  const WsLayout *L;
  int T, H, E, k;
  cudaStream_t s;
  const void *norm_w = nullptr; float eps = 0.f; void *x_norm_out = nullptr;   // one-token router only
  template <typename TA> int run() {
    RouterArgs<TA> a;
    a.x = (const TA *)x;
    a.w = (const TA *)w;
    a.idx_out = idx;
    a.w_out = (TA *)wout;
    a.logits_out = (TA *)logits;
    a.logits_ws = ws_ptr<float>(ws, L->logits);
    a.tile_cnt = ws_ptr<int>(ws, L->router_cnt);
    a.T = T; a.H = H; a.E = E; a.k = k;
    a.norm_w = (const TA *)norm_w; a.eps = eps; a.x_norm_out = (TA *)x_norm_out;
    if constexpr (sizeof(TA) == 2) {
      // decode-sized call: one thread-block cluster, no global synchronisation
      if (T <= kClusterMaxTFast && E <= kClusterMaxE && H / 8 <= 32 * 8 && (H / 8) % 32 == 0 && k <= 32) {
        a.pp = plan_ptrs(ws, *L);
        a.TB = T;
        a.n_ttiles = 1;
        a.n_etiles = kClusterCTAs;
        const dim3 grid(kClusterCTAs), block(kRouterThreads);
        if (T == 1 && k <= kT1MaxK) {
          if (norm_w != nullptr)
            return launch_cluster_pdl(k1_router_t1<TA, true>, grid, dim3(kT1Threads), (size_t)H * sizeof(TA),
                                      kClusterCTAs, s, "k1_router launch", a);
          return launch_cluster_pdl(k1_router_t1<TA, false>, grid, dim3(kT1Threads), (size_t)H * sizeof(TA),
                                    kClusterCTAs, s, "k1_router launch", a);
        }
        const size_t smem = std::max((size_t)T * H * sizeof(TA), plan_smem(kRouterWarps, E));
        switch (T <= 1 ? 1 : T <= 2 ? 2 : T <= 4 ? 4 : 8) {
          case 1: return launch_cluster_pdl(k1_router_cluster<TA, 1>, grid, block, smem, kClusterCTAs, s, "k1_router launch", a);
          case 2: return launch_cluster_pdl(k1_router_cluster<TA, 2>, grid, block, smem, kClusterCTAs, s, "k1_router launch", a);
          case 4: return launch_cluster_pdl(k1_router_cluster<TA, 4>, grid, block, smem, kClusterCTAs, s, "k1_router launch", a);
          default: return launch_cluster_pdl(k1_router_cluster<TA, 8>, grid, block, smem, kClusterCTAs, s, "k1_router launch", a);
        }
      }
      // every other 16-bit call: tensor-core logits, one cluster per 16 tokens
      // (64 for large calls: a quarter of the CTAs and of the weight re-reads)
      const int nt64 = (E + 63) / 64;
      const int NT = nt64 <= 1 ? 1 : nt64 <= 2 ? 2 : nt64 <= 4 ? 4 : nt64 <= 8 ? 8 : 16;
      const int MT = (T > 512 && NT <= 4) ? 4 : 1;
      a.pp = plan_ptrs(ws, *L);
      a.TB = kTcTile * MT;
      a.n_ttiles = (T + a.TB - 1) / a.TB;
      a.n_etiles = kClusterCTAs;
      if (a.n_ttiles > 65535) return fail(TM_ERR_UNSUPPORTED, "too many tokens for one router call (%d)", T);
      const dim3 grid(kClusterCTAs, a.n_ttiles), block(kRouterThreads);
      int rc;
#define TM_ROUTER_TC(nt_, mt_)                                                                              \
  rc = launch_cluster_pdl(k1_router_tc<TA, nt_, mt_>, grid, block, router_tc_smem<nt_, mt_>(E), kClusterCTAs, s, \
                          "k1_router_tc launch", a)
      if (MT == 4) {
        switch (NT) {
          case 1: TM_ROUTER_TC(1, 4); break;
          case 2: TM_ROUTER_TC(2, 4); break;
          default: TM_ROUTER_TC(4, 4); break;
        }
      } else {
        switch (NT) {
          case 1: TM_ROUTER_TC(1, 1); break;
          case 2: TM_ROUTER_TC(2, 1); break;
          case 4: TM_ROUTER_TC(4, 1); break;
          case 8: TM_ROUTER_TC(8, 1); break;
          default: TM_ROUTER_TC(16, 1); break;
        }
      }
#undef TM_ROUTER_TC
      if (rc || a.n_ttiles == 1) return rc;
      int ctas, units;
      plan_scatter_grid(T, &ctas, &units);
      return launch_pdl(k1_plan_scatter, dim3(ctas), dim3(kScatterThreads), plan_scatter_smem(E), s,
                        "k1_plan_scatter launch", (const int64_t *)idx, T, k, E, units, a.pp);
    } else {
      return run_fp32(a);
    }
  }
  int run_fp32(RouterArgs<float> &a) {
    if (T <= 8) { a.TB = T; a.EPW = 1; }
    else { a.TB = 16; a.EPW = 4; }
    // keep the token tile within 96 KB of shared memory
    while (a.TB > 1 && (size_t)a.TB * H * sizeof(float) > 96 * 1024) a.TB /= 2;
    a.n_ttiles = (T + a.TB - 1) / a.TB;
    const int ew = a.EPW * kRouterWarps;
    a.n_etiles = (E + ew - 1) / ew;
    if (a.n_ttiles > kMaxTokenTiles)
      return fail(TM_ERR_UNSUPPORTED, "too many tokens for one router call (%d)", T);
    a.pp = plan_ptrs(ws, *L);
    const size_t smem = std::max((size_t)a.TB * H * sizeof(float), plan_smem(kRouterWarps, E));
    const dim3 grid(a.n_etiles, a.n_ttiles), block(kRouterThreads);
    switch (a.TB <= 1 ? 1 : a.TB <= 2 ? 2 : a.TB <= 4 ? 4 : a.TB <= 8 ? 8 : 16) {
      case 1: return launch_pdl(k1_router<float, 1>, grid, block, smem, s, "k1_router launch", a);
      case 2: return launch_pdl(k1_router<float, 2>, grid, block, smem, s, "k1_router launch", a);
      case 4: return launch_pdl(k1_router<float, 4>, grid, block, smem, s, "k1_router launch", a);
      case 8: return launch_pdl(k1_router<float, 8>, grid, block, smem, s, "k1_router launch", a);
      default: return launch_pdl(k1_router<float, 16>, grid, block, smem, s, "k1_router launch", a);
    }
  }
};

}  // namespace tmoe

using namespace tmoe;

extern "C" int tm_router_topk(const void *x, int64_t tokens, int hidden, int act_dtype,
                              const void *router_w, int n_experts, int top_k, int64_t *topk_idx,
                              void *topk_w, void *logits_out, void *ws, int64_t ws_bytes,
                              void *stream) {
  TM_REQUIRE(x && router_w && topk_idx && topk_w, "null pointer");
  TM_REQUIRE(hidden > 0 && hidden % 128 == 0, "hidden (%d) must be a positive multiple of 128", hidden);
  TM_REQUIRE(n_experts <= 32 * kMaxExpertsPerLane, "n_experts %d > %d", n_experts, 32 * kMaxExpertsPerLane);
  TM_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= n_experts, "top_k %d must be in [1, min(32, n_experts %d)]", top_k, n_experts);
  TM_REQUIRE(aligned(x, 16) && aligned(router_w, 16), "x and router_w must be 16-byte aligned");
  WsLayout L;
  // the router only needs the header + logits + plan regions; expert sizes do not matter
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, 0, 0, &L);
  if (rc) return rc;
  RouterLaunch f{x, router_w, topk_idx, topk_w, logits_out, ws, &L, (int)tokens, hidden, n_experts, top_k,
                 as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_rmsnorm_router_topk(const void *x, int hidden, int act_dtype, const void *norm_w, float eps,
                                      void *x_norm_out, const void *router_w, int n_experts, int top_k,
                                      int64_t *topk_idx, void *topk_w, void *logits_out, void *ws, int64_t ws_bytes,
                                      void *stream) {
  TM_REQUIRE(x && norm_w && x_norm_out && router_w && topk_idx && topk_w, "null pointer");
  TM_REQUIRE(act_dtype == TM_DTYPE_BF16 || act_dtype == TM_DTYPE_F16, "16-bit activations only");
  TM_REQUIRE(hidden % 256 == 0 && hidden >= 256 && hidden <= 2048, "hidden %d must be a multiple of 256 up to 2048",
             hidden);
  TM_REQUIRE(n_experts >= 1 && n_experts <= kClusterMaxE && top_k >= 1 && top_k <= kT1MaxK && top_k <= n_experts,
             "n_experts %d / top_k %d outside the one-token router (E <= %d, k <= %d)", n_experts, top_k,
             kClusterMaxE, kT1MaxK);
  TM_REQUIRE(aligned(x, 16) && aligned(router_w, 16) && aligned(x_norm_out, 16) && aligned(norm_w, 2),
             "x, router_w and x_norm_out must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, 1, n_experts, top_k, hidden, 0, 0, &L);
  if (rc) return rc;
  RouterLaunch f{x, router_w, topk_idx, topk_w, logits_out, ws, &L, 1, hidden, n_experts, top_k, as_stream(stream)};
  f.norm_w = norm_w;
  f.eps = eps;
  f.x_norm_out = x_norm_out;
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_route_plan(const int64_t *topk_idx, int64_t tokens, int top_k, int n_experts,
                             void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(topk_idx, "null topk_idx");
  TM_REQUIRE(n_experts <= 512, "n_experts %d > 512 for tm_route_plan", n_experts);
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, 128, 0, 0, &L);
  if (rc) return rc;
  PlanPtrs pp = plan_ptrs(ws, L);
  if (tokens * top_k > 2048) {  // many pairs: counts per 16-token unit, then one CTA per range of units
    const int n_units = (int)((tokens + kUnitTokens - 1) / kUnitTokens);
    int rc = launch_pdl(k1_plan_hist, dim3(n_units), dim3(256), sizeof(int) * (size_t)n_experts, as_stream(stream),
                        "k1_plan_hist launch", topk_idx, (int)tokens, top_k, n_experts, pp);
    if (rc) return rc;
    int ctas, units;
    plan_scatter_grid(tokens, &ctas, &units);
    return launch_pdl(k1_plan_scatter, dim3(ctas), dim3(kScatterThreads), plan_scatter_smem(n_experts),
                      as_stream(stream), "k1_plan_scatter launch", topk_idx, (int)tokens, top_k, n_experts, units, pp);
  }
  const int threads = 1024;
  const size_t smem = plan_smem(threads / 32, n_experts);
  return launch_pdl(k1_plan_only, dim3(1), dim3(threads), smem, as_stream(stream), "k1_plan_only launch",
                    topk_idx, (int)tokens, top_k, n_experts, pp);
}

// K1: fused router (logits GEMV + fp32 softmax + top-k + renormalisation) and
// the routing plan (histogram, offsets, active experts, stable permutation).
//
// Reference: RouterExecutor.compute_routing (execution/router.py:15-42) and the
// implicit grouping in MoEExecutor.execute_layer (execution/moe.py:132,164-165):
// experts ascending (torch.unique), tokens ascending within an expert
// (torch.where over [T, k] in row-major order).
#include "tm_common.cuh"

namespace tmoe {

constexpr int kRouterThreads = 256;  // 8 warps
constexpr int kMaxExpertsPerLane = 32;  // E <= 1024

struct PlanPtrs {
  uint32_t *status;
  int *meta;
  int *counts;    // [E]
  int *offsets;   // [E+1]
  int *act_list;  // [E]
  int *slot_token, *slot_pair, *pair_slot;  // [P]
  int *k2_cnt;    // [(E+1)*rg_max]
  int *k3_cnt;    // [H/32]
  int k2_cnt_n, k3_cnt_n;
};

static PlanPtrs plan_ptrs(void *ws, const WsLayout &L) {
  PlanPtrs p;
  p.status = ws_ptr<uint32_t>(ws, L.status);
  p.meta = ws_ptr<int>(ws, L.meta);
  p.counts = ws_ptr<int>(ws, L.counts);
  p.offsets = ws_ptr<int>(ws, L.offsets);
  p.act_list = ws_ptr<int>(ws, L.act_list);
  p.slot_token = ws_ptr<int>(ws, L.slot_token);
  p.slot_pair = ws_ptr<int>(ws, L.slot_pair);
  p.pair_slot = ws_ptr<int>(ws, L.pair_slot);
  p.k2_cnt = ws_ptr<int>(ws, L.k2_cnt);
  p.k3_cnt = ws_ptr<int>(ws, L.k3_cnt);
  p.k2_cnt_n = (L.n_experts + 1) * kMaxRG;
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

// Build the routing plan from idx [T, k] (int64).  Whole block; `sm` needs
// (nwarps * E + 2 * E + 64) ints of shared memory.
__device__ void plan_build(const int64_t *__restrict__ idx, int T, int k, int E, const PlanPtrs &pp,
                           int *sm) {
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, nw = blockDim.x >> 5;
  const int P = T * k;
  int *hist = sm;                    // [nw][E]
  int *cnt = sm + nw * E;            // [E]
  int *flag = cnt + E;               // [E]
  int *tmp = flag + E;               // [33]
  for (int i = tid; i < nw * E; i += blockDim.x) hist[i] = 0;
  // the expert kernels' completion counters are zeroed for the next phases
  for (int i = tid; i < pp.k2_cnt_n; i += blockDim.x) pp.k2_cnt[i] = 0;
  for (int i = tid; i < pp.k3_cnt_n; i += blockDim.x) pp.k3_cnt[i] = 0;
  __syncthreads();
  const int lo = (int)((int64_t)w * P / nw), hi = (int)((int64_t)(w + 1) * P / nw);
  bool bad = false;
  for (int base = lo; base < hi; base += 32) {
    const int p = base + lane;
    if (p < hi) {
      const int64_t e = idx[p];
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
    flag[e] = run > 0 ? 1 : 0;
    pp.counts[e] = run;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) pp.offsets[e] = cnt[e];  // scanned below
  __syncthreads();
  const int total = block_excl_scan(cnt, E, tmp);
  const int n_active = block_excl_scan(flag, E, tmp);
  for (int e = tid; e < E; e += blockDim.x) {
    const int c = pp.offsets[e];
    pp.offsets[e] = cnt[e];
    if (c > 0) pp.act_list[flag[e]] = e;
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
      const int64_t v = idx[p];
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
};

// Dot products of router rows with the staged tokens.  Lane covers 16-byte
// vectors c*32+lane of the row (V act values each).
template <typename TA>
__device__ __forceinline__ void router_rows(const RouterArgs<TA> &a, const float *xs, int t0, int nt,
                                            int e_begin, int e_end) {
  constexpr int V = 16 / sizeof(TA);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nvec = a.H / V;  // 16-byte vectors per row
  for (int e = e_begin + w; e < e_end; e += kRouterThreads / 32) {
    const uint4 *row = reinterpret_cast<const uint4 *>(a.w + (int64_t)e * a.H);
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.f;
    for (int v = lane; v < nvec; v += 32) {
      const uint4 q = __ldg(row + v);
      const TA *qe = reinterpret_cast<const TA *>(&q);
      float wf[V];
#pragma unroll
      for (int i = 0; i < V; ++i) wf[i] = Act<TA>::to_f(qe[i]);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        if (j < nt) {
          const float *xr = xs + (int64_t)j * a.H + v * V;
#pragma unroll
          for (int i = 0; i < V; ++i) acc[j] = fmaf(wf[i], xr[i], acc[j]);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
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
}

// softmax(fp32) + top-k (value desc, lower id first on ties) + renormalise, one warp per token.
template <typename TA>
__device__ void router_topk_token(const RouterArgs<TA> &a, int t) {
  const int lane = threadIdx.x & 31;
  const float *lg = a.logits_ws + (int64_t)t * a.E;
  const int per = (a.E + 31) / 32;
  float v[kMaxExpertsPerLane];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = i * 32 + lane;
    v[i] = (i < per && e < a.E) ? ld_cg(lg + e) : -INFINITY;
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxExpertsPerLane; ++i) {
    const int e = i * 32 + lane;
    if (i < per && e < a.E) s += __expf(v[i] - m);
  }
  s = warp_sum(s);
  unsigned taken = 0;  // bit i: v[i] already selected
  float psel[32];
  int esel[32];
  float psum = 0.f;
  for (int r = 0; r < a.k; ++r) {
    // lane-local best: largest value, then smallest expert id (smallest i)
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxExpertsPerLane; ++i) {
      const int e = i * 32 + lane;
      if (i < per && e < a.E && !(taken & (1u << i))) {
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
    psel[r] = p;
    esel[r] = be;
    psum += p;
  }
  if (lane == 0) {
    for (int r = 0; r < a.k; ++r) {
      a.idx_out[(int64_t)t * a.k + r] = esel[r];
      a.w_out[(int64_t)t * a.k + r] = Act<TA>::from_f(psel[r] / psum);
    }
  }
}

template <typename TA>
__global__ void __launch_bounds__(kRouterThreads) k1_router(RouterArgs<TA> a) {
  extern __shared__ float xs[];  // [TB][H] fp32, reused by the plan phase
  __shared__ int s_flag;
  const int et = blockIdx.x, tt = blockIdx.y;
  const int t0 = tt * a.TB;
  const int nt = min(a.TB, a.T - t0);
  // stage the token tile as fp32
  for (int i = threadIdx.x; i < nt * a.H; i += blockDim.x) {
    const int j = i / a.H, c = i % a.H;
    xs[i] = Act<TA>::to_f(a.x[(int64_t)(t0 + j) * a.H + c]);
  }
  __syncthreads();
  const int e_begin = et * a.EPW * (kRouterThreads / 32);
  const int e_end = min(a.E, e_begin + a.EPW * (kRouterThreads / 32));
  router_rows<TA>(a, xs, t0, nt, e_begin, e_end);
  // the last expert tile of this token tile finishes the tokens
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&a.tile_cnt[tt], 1);
    s_flag = (prev == a.n_etiles - 1);
    if (s_flag) a.tile_cnt[tt] = 0;
  }
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  for (int j = threadIdx.x >> 5; j < nt; j += kRouterThreads / 32) router_topk_token<TA>(a, t0 + j);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&a.tile_cnt[kMaxTokenTiles], 1);
    s_flag = (prev == a.n_ttiles - 1);
    if (s_flag) a.tile_cnt[kMaxTokenTiles] = 0;
  }
  __syncthreads();
  if (!s_flag) return;
  __threadfence();
  plan_build(a.idx_out, a.T, a.k, a.E, a.pp, reinterpret_cast<int *>(xs));
}

__global__ void __launch_bounds__(1024) k1_plan_only(const int64_t *idx, int T, int k, int E, PlanPtrs pp) {
  extern __shared__ int sm[];
  plan_build(idx, T, k, E, pp, sm);
}

static size_t plan_smem(int nwarps, int E) { return sizeof(int) * ((size_t)nwarps * E + 2 * E + 64); }

struct RouterLaunch {
  const void *x, *w;
  int64_t *idx;
  void *wout, *logits;
  void *ws;
  const WsLayout *L;
  int T, H, E, k;
  cudaStream_t s;
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
    if (T <= 8) { a.TB = T; a.EPW = 1; }
    else { a.TB = 16; a.EPW = 4; }
    // keep the fp32 token tile within 160 KB of shared memory
    while (a.TB > 1 && (size_t)a.TB * H * 4 > 160 * 1024) a.TB /= 2;
    a.n_ttiles = (T + a.TB - 1) / a.TB;
    const int ew = a.EPW * (kRouterThreads / 32);
    a.n_etiles = (E + ew - 1) / ew;
    if (a.n_ttiles > kMaxTokenTiles)
      return fail(TM_ERR_UNSUPPORTED, "too many tokens for one router call (%d)", T);
    a.pp = plan_ptrs(ws, *L);
    size_t smem = std::max((size_t)a.TB * H * 4, plan_smem(kRouterThreads / 32, E));
    if (smem > 48 * 1024) {
      cudaError_t e = cudaFuncSetAttribute(k1_router<TA>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return cuda_check(e, "router smem attribute");
    }
    dim3 grid(a.n_etiles, a.n_ttiles);
    k1_router<TA><<<grid, kRouterThreads, smem, s>>>(a);
    TM_LAUNCH_CHECK("k1_router launch");
    return TM_OK;
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
  TM_REQUIRE(top_k <= 32, "top_k %d > 32", top_k);
  TM_REQUIRE(aligned(x, 16) && aligned(router_w, 16), "x and router_w must be 16-byte aligned");
  WsLayout L;
  // the router only needs the header + logits + plan regions; expert sizes do not matter
  int rc = ws_check(ws, ws_bytes, tokens, n_experts, top_k, hidden, 0, 0, &L);
  if (rc) return rc;
  RouterLaunch f{x, router_w, topk_idx, topk_w, logits_out, ws, &L, (int)tokens, hidden, n_experts, top_k,
                 as_stream(stream)};
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
  const int threads = 1024;
  const size_t smem = plan_smem(threads / 32, n_experts);
  cudaError_t e = cudaFuncSetAttribute(k1_plan_only, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_check(e, "plan smem attribute");
  k1_plan_only<<<1, threads, smem, as_stream(stream)>>>(topk_idx, (int)tokens, top_k, n_experts, pp);
  TM_LAUNCH_CHECK("k1_plan_only launch");
  return TM_OK;
}

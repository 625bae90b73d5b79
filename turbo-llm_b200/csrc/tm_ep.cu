// Expert parallelism over NVLink peer memory: one MoE layer with its experts
// sharded over the ranks of a node (one process per GPU), tokens dispatched
// to the expert owners and the outputs returned, with no collective library
// and no host synchronisation on the data path.
//
// The reference runs batch 1 on one device (runtime/engine.py:103-107,158)
// and has no expert parallelism; per token the arithmetic is that of
// MoEExecutor.execute_layer (execution/moe.py:99-208).
//
// Every rank allocates one buffer of identical layout (EpLayout) and maps its
// peers' buffers through CUDA IPC.  One layer call on a rank, in stream order:
//
//   source   tm_router_topk          top-k + routing plan (slots in expert order,
//                                    so each owner's rows are one slot range)
//            ep_dispatch             rows and {local expert, source slot} go
//                                    straight into each owner's receive region
//                                    (peer stores); the last CTA per owner
//                                    publishes the row count and the call's
//                                    epoch in the owner's arrival flag
//   owner    ep_owner_plan           bounded wait for every source's flag, then
//                                    the routing plan of the received rows
//            gate/up + down          tcgen05 grouped GEMMs over the received rows
//                                    (FP8 K7 for bf16, K4 for fp16)
//            ep_return               each output row back into its source's
//                                    return region at its source slot; then the
//                                    return flags
//   source   ep_wait_returns         bounded wait for every owner; advances the
//                                    epoch
//            tm_combine_slots        weighted sum in top-k order (+ residual)
//
// One region per kind suffices (no double buffering): a source dispatches
// call n+1 only after its combine of call n saw every owner's return flag,
// and an owner raises that flag after its last read of the rows, meta and
// counts of call n; an owner writes a source's return region of call n+1
// only after that source's dispatch of call n+1, which follows its combine of
// call n.  The epoch (calls completed) lives in device memory, so the whole
// sequence can be captured in a CUDA graph and replayed.
//
// Every wait is bounded in wall time (default 2 s); on expiry the kernel sets
// TM_STATUS_TIMEOUT in the context's status word and returns, so a missing
// peer costs an error, never a hung GPU.  An owner that gave up waiting for a
// source processes nothing and tags its return flags (kEpFailTag); every
// source that sees the tag sets TM_STATUS_PEER_FAILED, so no rank takes the
// stale rows of an earlier call for this call's outputs with a clean status.
// After either bit the context's regions may still receive late rows of the
// failed call: close and recreate the context before its next call.  No TMA, no multicast: peer memory
// is read and written with plain loads and stores only.
#include <new>

#include "tm_common.cuh"

namespace tmoe {

constexpr int kEpMaxRanks = TM_EP_MAX_RANKS;
constexpr int kEpThreads = 256;
constexpr int kEpWarps = kEpThreads / 32;
constexpr int kEpCopyCTAs = 296;      // row copies: two CTAs per SM, one warp per row
constexpr int kEpRowVecs = 8;         // 16-byte vectors a lane keeps in flight per row (H <= 2048 bf16: all)
constexpr uint64_t kEpDefaultTimeoutNs = 2000000000ull;
constexpr uint64_t kEpFailTag = 1ull << 63;   // in a return flag: the owner gave up on this call

struct EpLayout {
  int64_t flags;   // uint64 [2][kEpMaxRanks]: [0][src] rows of src arrived, [1][owner] outputs of owner returned
  int64_t counts;  // int32 [kEpMaxRanks]: rows received from each source
  int64_t rows;    // act [G][cap][H]: received token rows, source-major
  int64_t meta;    // int2 [G][cap]: {local expert, source slot} of each received row
  int64_t ret;     // act [pmax][H]: outputs for this rank's slots, written by the owners
  int64_t epoch;   // uint64, local: calls completed
  int64_t status;  // uint32, local: TM_STATUS_* bits
  int64_t owner_fail;  // uint32, local: 1 when this call's owner plan gave up waiting for a source
  int64_t done;    // int32 [kEpMaxRanks + 1], local: CTA completion counters
  int64_t total;
};

static EpLayout ep_layout(int G, int64_t cap, int64_t pmax, int H, int act_bytes) {
  EpLayout L;
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    const int64_t o = off;
    off = (off + bytes + 255) / 256 * 256;
    return o;
  };
  L.flags = take(2 * kEpMaxRanks * 8);
  L.counts = take(kEpMaxRanks * 4);
  L.rows = take((int64_t)G * cap * H * act_bytes);
  L.meta = take((int64_t)G * cap * 8);
  L.ret = take(pmax * H * act_bytes);
  L.epoch = take(8);
  L.status = take(4);
  L.owner_fail = take(4);
  L.done = take((kEpMaxRanks + 1) * 4);
  L.total = off;
  return L;
}

// What the kernels see of a context (passed by value).
struct EpDev {
  char *peer[kEpMaxRanks];  // every rank's buffer in this process's address space (own one included)
  char *local;
  EpLayout L;
  int rank, G, E_loc, H;
  int64_t cap, pmax;
  uint64_t timeout_ns;
};

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t *p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t *p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(int *p, int v) {
  asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint64_t ep_now_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Wait until (*flag & mask) == want for at most timeout_ns of wall time; the
// value seen last goes to *seen.
__device__ bool ep_wait_flag(const uint64_t *flag, uint64_t want, uint64_t timeout_ns, uint64_t mask = ~0ull,
                             uint64_t *seen = nullptr) {
  uint64_t v = ld_acquire_sys(flag);
  bool ok = (v & mask) == want;
  if (!ok) {
    const uint64_t t0 = ep_now_ns();
    while (true) {
      v = ld_acquire_sys(flag);
      if ((v & mask) == want) { ok = true; break; }
      if (ep_now_ns() - t0 > timeout_ns) break;
      __nanosleep(100);
    }
  }
  if (seen) *seen = v;
  return ok;
}
__device__ __forceinline__ uint64_t ep_next(const EpDev &d) {
  return *reinterpret_cast<volatile uint64_t *>(d.local + d.L.epoch) + 1;
}

// One warp copies one row of nv 16-byte vectors (local or peer memory): every
// load of a batch is issued before its stores.
__device__ __forceinline__ void ep_copy_row(uint4 *dst, const uint4 *src, int nv, int lane) {
  for (int b = 0; b < nv; b += 32 * kEpRowVecs) {
    uint4 v[kEpRowVecs];
#pragma unroll
    for (int u = 0; u < kEpRowVecs; ++u) {
      const int i = b + u * 32 + lane;
      if (i < nv) v[u] = __ldcg(src + i);
    }
#pragma unroll
    for (int u = 0; u < kEpRowVecs; ++u) {
      const int i = b + u * 32 + lane;
      if (i < nv) dst[i] = v[u];
    }
  }
}

// Source: send the rows of every owner's slot range, one warp per row.
// grid (CTAs per owner, G).
template <typename TA>
__global__ void __launch_bounds__(kEpThreads) ep_dispatch(EpDev d, const TA *x, const int64_t *idx,
                                                          const int *offsets, const int *slot_token,
                                                          const int *slot_pair) {
  const int tid = threadIdx.x, o = blockIdx.y, lane = tid & 31;
  const uint64_t ep = ep_next(d);
  const int s0 = __ldcg(offsets + o * d.E_loc), s1 = __ldcg(offsets + (o + 1) * d.E_loc);
  int n = s1 - s0;
  if (n > d.cap || n < 0) {  // cannot happen for a valid plan (top-k ids are distinct per token)
    if (tid == 0) atomicOr(reinterpret_cast<uint32_t *>(d.local + d.L.status), TM_STATUS_BAD_EXPERT_ID);
    n = 0;
  }
  TA *dst_rows = reinterpret_cast<TA *>(d.peer[o] + d.L.rows) + (int64_t)d.rank * d.cap * d.H;
  int2 *dst_meta = reinterpret_cast<int2 *>(d.peer[o] + d.L.meta) + (int64_t)d.rank * d.cap;
  const int nv = d.H * (int)sizeof(TA) / 16;
  for (int i = blockIdx.x * kEpWarps + (tid >> 5); i < n; i += gridDim.x * kEpWarps) {
    const int s = s0 + i;
    const int t = __ldcg(slot_token + s);
    ep_copy_row(reinterpret_cast<uint4 *>(dst_rows + (int64_t)i * d.H),
                reinterpret_cast<const uint4 *>(x + (int64_t)t * d.H), nv, lane);
    if (lane == 0) {
      const int e = (int)__ldcg(idx + __ldcg(slot_pair + s));
      dst_meta[i] = make_int2(e - o * d.E_loc, s);
    }
  }
  // the CTA's stores are ordered before thread 0's system-scope fence by the
  // barrier (fence cumulativity): one fence per CTA, not per thread
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    int *done = reinterpret_cast<int *>(d.local + d.L.done) + o;
    if (atomicAdd(done, 1) == (int)gridDim.x - 1) {
      atomicExch(done, 0);
      __threadfence_system();
      st_relaxed_sys(reinterpret_cast<int *>(d.peer[o] + d.L.counts) + d.rank, n);
      st_release_sys(reinterpret_cast<uint64_t *>(d.peer[o] + d.L.flags) + d.rank, ep);
    }
  }
}

struct OwnerPlan {
  int *meta, *counts, *offsets, *act_list;
  int4 *act_rec;
  int *slot_token, *slot_pair, *pair_slot;
};

// Owner: wait for every source, then the routing plan of the received rows
// (one pair per row, k = 1): experts ascending, then source, then arrival
// order; slot_token = slot_pair = the row's index in the receive region;
// capacity rows nobody filled get pair_slot -1.  One CTA of 1024 threads;
// dynamic shared memory (32 * E_loc + 3 * E_loc + 64) ints.
__global__ void __launch_bounds__(1024) ep_owner_plan(EpDev d, OwnerPlan pp) {
  extern __shared__ int osm[];
  __shared__ int s_pre[kEpMaxRanks + 1];
  __shared__ int s_fail;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, nw = blockDim.x >> 5;
  const int E = d.E_loc, G = d.G;
  const uint64_t ep = ep_next(d);
  uint32_t *status = reinterpret_cast<uint32_t *>(d.local + d.L.status);
  if (tid == 0) s_fail = 0;
  __syncthreads();
  int cnt_g = 0;
  if (tid < G) {
    const uint64_t *flag = reinterpret_cast<const uint64_t *>(d.local + d.L.flags) + tid;
    if (ep_wait_flag(flag, ep, d.timeout_ns)) {
      cnt_g = __ldcg(reinterpret_cast<const int *>(d.local + d.L.counts) + tid);
      if (cnt_g < 0 || cnt_g > d.cap) {
        atomicOr(status, TM_STATUS_BAD_EXPERT_ID);
        cnt_g = 0;
      }
    } else {
      atomicOr(&s_fail, 1);
    }
  }
  // source counts -> prefix (warp 0 holds them)
  if (w == 0) {
    int incl = lane < G ? cnt_g : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane < G) s_pre[lane + 1] = incl;
    if (lane == 0) s_pre[0] = 0;
  }
  int *hist = osm;                 // [nw][E]
  int *cnt = hist + nw * E;        // [E] counts, then offsets
  int *flg = cnt + E;              // [E] active flag, then active index
  int *cnt0 = flg + E;             // [E]
  int *tmp = cnt0 + E;             // [33]
  for (int i = tid; i < nw * E; i += blockDim.x) hist[i] = 0;
  const int64_t rows = (int64_t)G * d.cap;
  for (int64_t r = tid; r < rows; r += blockDim.x) pp.pair_slot[r] = -1;
  __syncthreads();
  if (tid == 0) *reinterpret_cast<volatile uint32_t *>(d.local + d.L.owner_fail) = s_fail ? 1u : 0u;
  if (s_fail) {
    if (tid == 0) atomicOr(status, TM_STATUS_TIMEOUT);
    if (tid < G + 1) s_pre[tid] = 0;  // process nothing
  }
  __syncthreads();
  const int R = s_pre[G];
  const int2 *meta = reinterpret_cast<const int2 *>(d.local + d.L.meta);
  auto row_of = [&](int p) -> int64_t {
    int g = 0;
    while (g + 1 < G && p >= s_pre[g + 1]) ++g;
    return (int64_t)g * d.cap + (p - s_pre[g]);
  };
  auto expert_of = [&](int64_t row) -> int {
    const int e = __ldcg(&meta[row].x);
    return (e >= 0 && e < E) ? e : -1;
  };
  const int lo = (int)((int64_t)w * R / nw), hi = (int)((int64_t)(w + 1) * R / nw);
  bool bad = false;
  for (int b = lo; b < hi; b += 32) {
    const int p = b + lane;
    if (p < hi) {
      const int e = expert_of(row_of(p));
      if (e >= 0) atomicAdd(&hist[w * E + e], 1);
      else bad = true;
    }
  }
  if (__any_sync(0xffffffffu, bad) && lane == 0) atomicOr(status, TM_STATUS_BAD_EXPERT_ID);
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    int run = 0;
    for (int j = 0; j < nw; ++j) {
      const int c = hist[j * E + e];
      hist[j * E + e] = run;
      run += c;
    }
    cnt[e] = run;
    cnt0[e] = run;
    flg[e] = run > 0 ? 1 : 0;
    pp.counts[e] = run;
  }
  __syncthreads();
  // exclusive scans of cnt and flg (E <= 1024: one element per thread)
  for (int pass = 0; pass < 2; ++pass) {
    int *a = pass == 0 ? cnt : flg;
    const int v = tid < E ? a[tid] : 0;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) tmp[w] = incl;
    __syncthreads();
    if (w == 0) {
      const int t = lane < nw ? tmp[lane] : 0;
      int ti = t;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, ti, o);
        if (lane >= o) ti += u;
      }
      if (lane < nw) tmp[lane] = ti - t;
      if (lane == 31) tmp[32] = ti;
    }
    __syncthreads();
    if (tid < E) a[tid] = tmp[w] + incl - v;
    if (pass == 0 && tid == 0) {
      pp.offsets[E] = tmp[32];
      pp.meta[kMetaPairs] = tmp[32];  // rows with a valid expert id (the slots)
    }
    if (pass == 1 && tid == 0) pp.meta[kMetaNActive] = tmp[32];
    __syncthreads();
  }
  for (int e = tid; e < E; e += blockDim.x) {
    const int c = cnt0[e];
    pp.offsets[e] = cnt[e];
    if (c > 0) {
      pp.act_list[flg[e]] = e;
      pp.act_rec[flg[e]] = make_int4(e, c, cnt[e], 0);
    }
    for (int j = 0; j < nw; ++j) hist[j * E + e] += cnt[e];
  }
  if (tid == 0) pp.meta[kMetaTokens] = (int)rows;
  __syncthreads();
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int b = lo; b < hi; b += 32) {
    const int p = b + lane;
    int64_t row = -1;
    int e = -1;
    if (p < hi) {
      row = row_of(p);
      e = expert_of(row);
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & lt_mask);
    if (e >= 0) {
      const int slot = hist[w * E + e] + rank;
      pp.slot_token[slot] = (int)row;
      pp.slot_pair[slot] = (int)row;
      pp.pair_slot[row] = slot;
    }
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) hist[w * E + e] += __popc(peers);
    __syncwarp();
  }
}

// Owner: every output row to its source's return region, then the flags
// (tagged with kEpFailTag when this call's owner plan gave up).
template <typename TA>
__global__ void __launch_bounds__(kEpThreads) ep_return(EpDev d, const TA *y, const int *slot_token,
                                                        const int *plan_meta) {
  const int tid = threadIdx.x, lane = tid & 31;
  const uint64_t ep = ep_next(d);
  const int R = __ldcg(plan_meta + kMetaPairs);
  const int nv = d.H * (int)sizeof(TA) / 16;
  const int2 *meta = reinterpret_cast<const int2 *>(d.local + d.L.meta);
  for (int s = blockIdx.x * kEpWarps + (tid >> 5); s < R; s += gridDim.x * kEpWarps) {
    const int row = __ldcg(slot_token + s);
    const int g = (int)(row / d.cap);
    const int src_slot = __ldcg(&meta[row].y);
    if (g < 0 || g >= d.G || src_slot < 0 || src_slot >= d.pmax) continue;  // not from a valid dispatch
    ep_copy_row(reinterpret_cast<uint4 *>(reinterpret_cast<TA *>(d.peer[g] + d.L.ret) + (int64_t)src_slot * d.H),
                reinterpret_cast<const uint4 *>(y + (int64_t)s * d.H), nv, lane);
  }
  __syncthreads();
  if (tid == 0) {
    __threadfence_system();
    int *done = reinterpret_cast<int *>(d.local + d.L.done) + kEpMaxRanks;
    if (atomicAdd(done, 1) == (int)gridDim.x - 1) {
      atomicExch(done, 0);
      __threadfence_system();
      const bool failed = *reinterpret_cast<volatile uint32_t *>(d.local + d.L.owner_fail) != 0u;
      const uint64_t v = failed ? (ep | kEpFailTag) : ep;
      for (int g = 0; g < d.G; ++g)
        st_release_sys(reinterpret_cast<uint64_t *>(d.peer[g] + d.L.flags) + kEpMaxRanks + d.rank, v);
    }
  }
}

// Source: wait for every owner's outputs, then count the call as done.  A
// return flag tagged kEpFailTag (the owner gave up on this call) sets
// TM_STATUS_PEER_FAILED: the rows that owner should have returned are stale.
__global__ void ep_wait_returns(EpDev d) {
  const int lane = threadIdx.x & 31;
  const uint64_t ep = ep_next(d);
  bool ok = true, peer_failed = false;
  if (lane < d.G) {
    uint64_t seen = 0;
    ok = ep_wait_flag(reinterpret_cast<const uint64_t *>(d.local + d.L.flags) + kEpMaxRanks + lane, ep,
                      d.timeout_ns, ~kEpFailTag, &seen);
    peer_failed = ok && (seen & kEpFailTag) != 0;
  }
  uint32_t *status = reinterpret_cast<uint32_t *>(d.local + d.L.status);
  if (!__all_sync(0xffffffffu, ok) && lane == 0) atomicOr(status, TM_STATUS_TIMEOUT);
  if (__any_sync(0xffffffffu, peer_failed) && lane == 0) atomicOr(status, TM_STATUS_PEER_FAILED);
  __syncwarp();
  if (lane == 0) *reinterpret_cast<volatile uint64_t *>(d.local + d.L.epoch) = ep;
}

}  // namespace tmoe

struct tm_ep_ctx {
  int device, rank, world, n_experts, e_loc, top_k, hidden, inter, act, act_bytes;
  int64_t max_tokens, cap, pmax;
  tmoe::EpLayout L;
  char *base;
  char *peer[tmoe::kEpMaxRanks];
  bool opened[tmoe::kEpMaxRanks];
  bool connected;
  uint64_t timeout_ns;
};

using namespace tmoe;

static int act_bytes_of(int act_dtype) { return act_dtype == TM_DTYPE_F32 ? 4 : 2; }

static EpDev ep_dev(const tm_ep_ctx *c) {
  EpDev d;
  for (int r = 0; r < kEpMaxRanks; ++r) d.peer[r] = r < c->world ? c->peer[r] : nullptr;
  d.local = c->base;
  d.L = c->L;
  d.rank = c->rank;
  d.G = c->world;
  d.E_loc = c->e_loc;
  d.H = c->hidden;
  d.cap = c->cap;
  d.pmax = c->pmax;
  d.timeout_ns = c->timeout_ns;
  return d;
}

// rows one source can send one owner: each token routes to distinct experts
static int64_t ep_cap(int64_t max_tokens, int top_k, int e_loc) {
  return max_tokens * (int64_t)(top_k < e_loc ? top_k : e_loc);
}

extern "C" int64_t tm_ep_buffer_bytes(int world, int64_t max_tokens, int n_experts, int top_k, int hidden,
                                      int act_dtype) {
  if (world < 1 || world > kEpMaxRanks || max_tokens < 1 || n_experts < world || n_experts % world || top_k < 1 ||
      hidden < 8)
    return fail(TM_ERR_INVALID, "bad expert-parallel shape");
  const int e_loc = n_experts / world;
  return ep_layout(world, ep_cap(max_tokens, top_k, e_loc), max_tokens * top_k, hidden, act_bytes_of(act_dtype))
      .total;
}

extern "C" int tm_ep_create(int rank, int world, int n_experts, int top_k, int hidden, int inter, int act_dtype,
                            int64_t max_tokens, void *handle_out, tm_ep_ctx **out) {
  TM_REQUIRE(out != nullptr && handle_out != nullptr, "null pointer");
  *out = nullptr;
  TM_REQUIRE(world >= 1 && world <= kEpMaxRanks && rank >= 0 && rank < world, "rank %d / world %d (at most %d)",
             rank, world, kEpMaxRanks);
  TM_REQUIRE(n_experts >= world && n_experts % world == 0, "%d experts do not shard over %d ranks", n_experts,
             world);
  TM_REQUIRE(top_k >= 1 && top_k <= 32 && top_k <= n_experts, "bad top_k %d", top_k);
  TM_REQUIRE(act_dtype == TM_DTYPE_BF16 || act_dtype == TM_DTYPE_F16, "act dtype must be bf16 or fp16");
  TM_REQUIRE(hidden % 256 == 0 && hidden > 0 && inter % 128 == 0 && inter > 0,
             "hidden %d (multiple of 256) / inter %d (multiple of 128) unsupported", hidden, inter);
  TM_REQUIRE(max_tokens >= 1 && max_tokens <= (1 << 20), "max_tokens %lld out of range", (long long)max_tokens);
  tm_ep_ctx *c = new (std::nothrow) tm_ep_ctx();
  if (!c) return fail(TM_ERR_INVALID, "out of host memory");
  int rc = cuda_check(cudaGetDevice(&c->device), "cudaGetDevice");
  if (rc) { delete c; return rc; }
  c->rank = rank; c->world = world; c->n_experts = n_experts; c->e_loc = n_experts / world;
  c->top_k = top_k; c->hidden = hidden; c->inter = inter; c->act = act_dtype;
  c->act_bytes = act_bytes_of(act_dtype);
  c->max_tokens = max_tokens;
  c->cap = ep_cap(max_tokens, top_k, c->e_loc);
  c->pmax = max_tokens * top_k;
  c->L = ep_layout(world, c->cap, c->pmax, hidden, c->act_bytes);
  c->timeout_ns = kEpDefaultTimeoutNs;
  rc = cuda_check(cudaMalloc(reinterpret_cast<void **>(&c->base), (size_t)c->L.total), "cudaMalloc (EP buffer)");
  if (rc) { delete c; return rc; }
  rc = cuda_check(cudaMemset(c->base, 0, (size_t)c->L.total), "cudaMemset (EP buffer)");
  if (!rc) {
    cudaIpcMemHandle_t h;
    rc = cuda_check(cudaIpcGetMemHandle(&h, c->base), "cudaIpcGetMemHandle");
    if (!rc) memcpy(handle_out, &h, sizeof(h) < TM_EP_HANDLE_BYTES ? sizeof(h) : TM_EP_HANDLE_BYTES);
  }
  if (rc) {
    cudaFree(c->base);
    delete c;
    return rc;
  }
  for (int r = 0; r < kEpMaxRanks; ++r) { c->peer[r] = nullptr; c->opened[r] = false; }
  c->peer[rank] = c->base;
  *out = c;
  return TM_OK;
}

extern "C" int tm_ep_connect(tm_ep_ctx *c, const void *handles) {
  TM_REQUIRE(c && handles, "null pointer");
  TM_REQUIRE(!c->connected, "context already connected");
  int rc = cuda_check(cudaSetDevice(c->device), "cudaSetDevice");
  if (rc) return rc;
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const char *>(handles) + (size_t)r * TM_EP_HANDLE_BYTES, sizeof(h));
    void *p = nullptr;
    rc = cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    if (rc) return rc;
    c->peer[r] = static_cast<char *>(p);
    c->opened[r] = true;
  }
  c->connected = true;
  return TM_OK;
}

extern "C" int tm_ep_connect_ptrs(tm_ep_ctx *c, void *const *peer_bases) {
  TM_REQUIRE(c && peer_bases, "null pointer");
  TM_REQUIRE(!c->connected, "context already connected");
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) continue;
    TM_REQUIRE(peer_bases[r] != nullptr && aligned(peer_bases[r], 256), "peer %d base missing or unaligned", r);
    c->peer[r] = static_cast<char *>(peer_bases[r]);
  }
  c->connected = true;
  return TM_OK;
}

extern "C" void *tm_ep_local_buffer(tm_ep_ctx *c) { return c ? c->base : nullptr; }

extern "C" int tm_ep_set_timeout(tm_ep_ctx *c, int64_t timeout_ns) {
  TM_REQUIRE(c && timeout_ns > 0, "bad arguments");
  c->timeout_ns = (uint64_t)timeout_ns;
  return TM_OK;
}

extern "C" int tm_ep_disconnect(tm_ep_ctx *c) {
  TM_REQUIRE(c, "null context");
  int rc = cuda_check(cudaSetDevice(c->device), "cudaSetDevice");
  if (!rc) rc = cuda_check(cudaDeviceSynchronize(), "cudaDeviceSynchronize");
  for (int r = 0; r < kEpMaxRanks; ++r) {
    if (c->opened[r]) {
      const int rc2 = cuda_check(cudaIpcCloseMemHandle(c->peer[r]), "cudaIpcCloseMemHandle");
      if (!rc) rc = rc2;
      c->opened[r] = false;
    }
    if (r != c->rank) c->peer[r] = nullptr;
  }
  c->connected = false;
  return rc;
}

extern "C" int tm_ep_destroy(tm_ep_ctx *c) {
  if (!c) return TM_OK;
  int rc = TM_OK;
  if (c->connected) rc = tm_ep_disconnect(c);
  cudaSetDevice(c->device);
  const int rc2 = cuda_check(cudaFree(c->base), "cudaFree (EP buffer)");
  delete c;
  return rc ? rc : rc2;
}

extern "C" int64_t tm_ep_owner_workspace_bytes(const tm_ep_ctx *c) {
  if (!c) return fail(TM_ERR_INVALID, "null context");
  return ws_layout((int64_t)c->world * c->cap, c->e_loc, 1, c->hidden, c->inter, 0).total;
}

extern "C" int tm_ep_status(tm_ep_ctx *c, uint32_t *host_status, void *stream) {
  TM_REQUIRE(c && host_status, "null pointer");
  cudaStream_t s = as_stream(stream);
  char *p = c->base + c->L.status;
  int rc = cuda_check(cudaMemcpyAsync(host_status, p, 4, cudaMemcpyDeviceToHost, s), "EP status copy");
  if (rc) return rc;
  rc = cuda_check(cudaStreamSynchronize(s), "EP status sync");
  if (rc) return rc;
  return cuda_check(cudaMemsetAsync(p, 0, 4, s), "EP status clear");
}

namespace tmoe {
struct EpDispatchLaunch {
  const tm_ep_ctx *c; const void *x; const int64_t *idx; const WsLayout *L; void *ws; cudaStream_t s;
  template <typename TA> int run() {
    if constexpr (sizeof(TA) != 2) {
      return fail(TM_ERR_UNSUPPORTED, "expert parallelism needs bf16 or fp16 activations");
    } else {
      const dim3 grid((kEpCopyCTAs + c->world - 1) / c->world, c->world);
      ep_dispatch<TA><<<grid, kEpThreads, 0, s>>>(ep_dev(c), (const TA *)x, idx, ws_ptr<int>(ws, L->offsets),
                                                  ws_ptr<int>(ws, L->slot_token), ws_ptr<int>(ws, L->slot_pair));
      TM_LAUNCH_CHECK("ep_dispatch launch");
      return TM_OK;
    }
  }
};
struct EpReturnLaunch {
  const tm_ep_ctx *c; const WsLayout *L; void *ws; cudaStream_t s;
  template <typename TA> int run() {
    if constexpr (sizeof(TA) != 2) {
      return fail(TM_ERR_UNSUPPORTED, "expert parallelism needs bf16 or fp16 activations");
    } else {
      ep_return<TA><<<kEpCopyCTAs, kEpThreads, 0, s>>>(ep_dev(c), ws_ptr<TA>(ws, L->ypart),
                                                        ws_ptr<int>(ws, L->slot_token), ws_ptr<int>(ws, L->meta));
      TM_LAUNCH_CHECK("ep_return launch");
      return TM_OK;
    }
  }
};
}  // namespace tmoe

extern "C" int tm_ep_dispatch(tm_ep_ctx *c, const void *x, int64_t tokens, const int64_t *topk_idx, void *ws,
                              int64_t ws_bytes, void *stream) {
  TM_REQUIRE(c && x && topk_idx, "null pointer");
  TM_REQUIRE(c->connected, "context not connected");
  TM_REQUIRE(tokens >= 1 && tokens <= c->max_tokens, "tokens %lld outside [1, %lld]", (long long)tokens,
             (long long)c->max_tokens);
  TM_REQUIRE(aligned(x, 16), "x must be 16-byte aligned");
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, c->n_experts, c->top_k, c->hidden, 0, 0, &L);
  if (rc) return rc;
  EpDispatchLaunch f{c, x, topk_idx, &L, ws, as_stream(stream)};
  return dispatch_act(c->act, f);
}

extern "C" int tm_ep_experts(tm_ep_ctx *c, const uint8_t *w13, const float *s13, const uint8_t *w2,
                             const float *s2, void *owner_ws, int64_t owner_ws_bytes, void *stream) {
  TM_REQUIRE(c && w13 && s13 && w2 && s2, "null pointer");
  TM_REQUIRE(c->connected, "context not connected");
  TM_REQUIRE(aligned(w13, 16) && aligned(w2, 16), "weights must be 16-byte aligned");
  const int64_t rows = (int64_t)c->world * c->cap;
  WsLayout L;
  int rc = ws_check(owner_ws, owner_ws_bytes, rows, c->e_loc, 1, c->hidden, c->inter, 0, &L);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  OwnerPlan pp;
  pp.meta = ws_ptr<int>(owner_ws, L.meta);
  pp.counts = ws_ptr<int>(owner_ws, L.counts);
  pp.offsets = ws_ptr<int>(owner_ws, L.offsets);
  pp.act_list = ws_ptr<int>(owner_ws, L.act_list);
  pp.act_rec = ws_ptr<int4>(owner_ws, L.act_rec);
  pp.slot_token = ws_ptr<int>(owner_ws, L.slot_token);
  pp.slot_pair = ws_ptr<int>(owner_ws, L.slot_pair);
  pp.pair_slot = ws_ptr<int>(owner_ws, L.pair_slot);
  const size_t smem = sizeof(int) * ((size_t)(32 + 3) * c->e_loc + 64);
  rc = ensure_smem(reinterpret_cast<const void *>(ep_owner_plan), smem);
  if (rc) return rc;
  ep_owner_plan<<<1, 1024, smem, s>>>(ep_dev(c), pp);
  TM_LAUNCH_CHECK("ep_owner_plan launch");
  // bf16: the FP8 tensor-core GEMMs (owners see ~16 rows per expert); fp16: the dequantising ones
  rc = c->act == TM_DTYPE_BF16
           ? f8_expert_outputs(c->base + c->L.rows, rows, c->hidden, c->inter, c->e_loc, 1, w13, s13, w2, s2, nullptr,
                               nullptr, nullptr, nullptr, nullptr, owner_ws, L, s)
           : prefill_expert_outputs(c->base + c->L.rows, rows, c->hidden, c->inter, c->e_loc, 1, c->act, w13, s13, w2,
                                    s2, owner_ws, L, s);
  if (rc) return rc;
  EpReturnLaunch f{c, &L, owner_ws, s};
  return dispatch_act(c->act, f);
}

extern "C" int tm_ep_combine(tm_ep_ctx *c, const void *topk_w, int64_t tokens, void *ws, int64_t ws_bytes,
                             const void *residual, void *out, void *stream) {
  TM_REQUIRE(c && topk_w && out, "null pointer");
  TM_REQUIRE(c->connected, "context not connected");
  TM_REQUIRE(tokens >= 1 && tokens <= c->max_tokens, "tokens %lld outside [1, %lld]", (long long)tokens,
             (long long)c->max_tokens);
  WsLayout L;
  int rc = ws_check(ws, ws_bytes, tokens, c->n_experts, c->top_k, c->hidden, 0, 0, &L);
  if (rc) return rc;
  cudaStream_t s = as_stream(stream);
  ep_wait_returns<<<1, 32, 0, s>>>(ep_dev(c));
  TM_LAUNCH_CHECK("ep_wait_returns launch");
  return tm_combine_slots(c->base + c->L.ret, topk_w, ws_ptr<int32_t>(ws, L.pair_slot), tokens, c->hidden,
                          c->top_k, c->act, residual, out, stream);
}

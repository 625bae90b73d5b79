// The rest of a Qwen3-MoE decode step around the MoE hot path: token
// embedding, RMSNorm, per-head q/k RMSNorm + rotary embedding + KV-cache
// append, one-token attention over the KV cache, and the LM head with the
// greedy argmax.  With tm_fp8_linear (q/k/v/o projections) and the MoE
// kernels they make one decode step that never leaves the device: the next
// token id is written to device memory and read by the next step's
// embedding, so a whole step can be replayed from one CUDA graph.
//
// Reference (the Hugging Face Qwen3-MoE modules the reference engine drives,
// runtime/engine.py:98-162, execution/layer_executor.py:137-170):
//   embed_tokens; input_layernorm / post_attention_layernorm / q_norm /
//   k_norm / norm (RMSNorm: fp32 variance, x * rsqrt(var + eps) rounded to the
//   act dtype, times the weight, rounded); apply_rotary_pos_emb
//   (q * cos + rotate_half(q) * sin, every product and the sum rounded to the
//   act dtype); scaled-dot-product attention over the cache (GQA); lm_head;
//   torch.argmax of the last position's logits (first index among equal
//   maxima).
//
// Layouts: KV cache of one layer [n_kv][max_len][head_dim] (act dtype), so the
// rows one KV head reads are contiguous; rotary table [max_len][2][head_dim]
// (cos, then sin) in the act dtype, computed by the host exactly as the
// reference does (inv_freq in fp32, position * inv_freq, cos/sin in fp32,
// rounded to the act dtype).
#include "tm_common.cuh"

#include <algorithm>
#include <mutex>

namespace tmoe {

constexpr int kHeadDim = 128;
constexpr int kAttnTile = 32;   // positions per shared-memory tile
constexpr int kHeadMaxAttnWarps = 16;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Four consecutive act values <-> floats.
template <typename TA> struct Vec4;
template <> struct Vec4<float> {
  static __device__ __forceinline__ void load(const float *p, float (&v)[4]) {
    const float4 r = *reinterpret_cast<const float4 *>(p);
    v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
  }
  static __device__ __forceinline__ void load_cg(const float *p, float (&v)[4]) {
    const float4 r = __ldcg(reinterpret_cast<const float4 *>(p));
    v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
  }
  static __device__ __forceinline__ void store(float *p, const float (&v)[4]) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <typename TA> struct Vec4Half {
  static __device__ __forceinline__ void unpack(uint2 r, float (&v)[4]) {
    const TA *h = reinterpret_cast<const TA *>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = Act<TA>::to_f(h[i]);
  }
  static __device__ __forceinline__ void load(const TA *p, float (&v)[4]) {
    unpack(*reinterpret_cast<const uint2 *>(p), v);
  }
  static __device__ __forceinline__ void load_cg(const TA *p, float (&v)[4]) {
    unpack(__ldcg(reinterpret_cast<const uint2 *>(p)), v);
  }
  static __device__ __forceinline__ void store(TA *p, const float (&v)[4]) {
    uint2 r;
    TA *h = reinterpret_cast<TA *>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = Act<TA>::from_f(v[i]);
    *reinterpret_cast<uint2 *>(p) = r;
  }
};
template <> struct Vec4<__half> : Vec4Half<__half> {};
template <> struct Vec4<__nv_bfloat16> : Vec4Half<__nv_bfloat16> {};

// 16-byte asynchronous global -> shared copy (L2 only; the cache rows were
// written by an earlier kernel of the step).
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

// ------------------------------------------------------------------ embed ----
// out[t] = table[ids[t]] (bf16 table -> act dtype, exact).  ids are read
// through L2: the previous step's argmax wrote them.
template <typename TO>
__global__ void __launch_bounds__(256) k8_embed(const int64_t *ids, const __nv_bfloat16 *table, int hidden,
                                                int64_t vocab, TO *out, uint32_t *status) {
  pdl_wait();
  pdl_trigger();
  const int t = blockIdx.x;
  const int64_t id = (int64_t)__ldcg(reinterpret_cast<const long long *>(ids) + t);
  TO *o = out + (int64_t)t * hidden;
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && status) atomicOr(status, TM_STATUS_BAD_TOKEN_ID);
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = Act<TO>::from_f(0.f);
    return;
  }
  const __nv_bfloat16 *row = table + id * hidden;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) o[i] = Act<TO>::from_f(__bfloat162float(row[i]));
}

// ---------------------------------------------------------------- RMSNorm ----
// One CTA per token: out = round(round(x * rsqrt(mean(x^2) + eps)) * w).
// Threads hold 4 consecutive elements (one 8- or 16-byte load), the row
// stays in registers between the sum of squares and the output (hidden <=
// 4096 with 256 threads).
template <typename TA>
__global__ void __launch_bounds__(256) k8_rmsnorm(const TA *x, const TA *w, int hidden, float eps, TA *out) {
  __shared__ float red[8];
  const int t = blockIdx.x, tid = threadIdx.x;
  float wv[4][4];
  for (int c = 0; c < 4; ++c) {   // the weights do not depend on the previous kernel
    const int i = (c * 256 + tid) * 4;
    if (i < hidden) Vec4<TA>::load(w + i, wv[c]);
  }
  pdl_wait();
  const TA *xr = x + (int64_t)t * hidden;
  float v[4][4];
  float ss = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int i = (c * 256 + tid) * 4;
    if (i < hidden) {
      Vec4<TA>::load_cg(xr + i, v[c]);
#pragma unroll
      for (int e = 0; e < 4; ++e) ss = fmaf(v[c][e], v[c][e], ss);
    }
  }
  pdl_trigger();
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) tot += red[i];
  const float r = rsqrtf(tot / (float)hidden + eps);
  TA *o = out + (int64_t)t * hidden;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int i = (c * 256 + tid) * 4;
    if (i < hidden) {
      float y[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) y[e] = Act<TA>::round(v[c][e] * r) * wv[c][e];
      Vec4<TA>::store(o + i, y);
    }
  }
}

// ------------------------------------------- q/k norm, RoPE, KV append ----
// qkv [T][(nh + 2 nkv) * 128]: q heads, then k heads, then v heads (the output
// of the fused q/k/v projection).  One warp per (token, head); lane j holds
// elements 4j..4j+3.  q heads: RMSNorm (q_norm) + rotary -> q_out [T][nh][128];
// k heads: RMSNorm (k_norm) + rotary -> k_cache[kvh][pos]; v heads -> v_cache.
// One head of the q/k norm + rotary step for one warp: lane j holds elements
// 4j..4j+3 in v; RMSNorm over the head (weight nw), then rotate_half with the
// cos/sin of position pos from the table (Qwen3MoeAttention's q_norm / k_norm
// and apply_rotary_pos_emb, rounded to the act dtype where they round).
template <typename TA>
__device__ __forceinline__ void qk_norm_rope(const float (&v)[4], const TA *nw, float eps, const TA *rope,
                                             int64_t pos, int lane, float (&out)[4]) {
  const int e0 = 4 * lane;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) ss = fmaf(v[i], v[i], ss);
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)kHeadDim + eps);
  float n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = Act<TA>::round(Act<TA>::round(v[i] * r) * Act<TA>::to_f(nw[e0 + i]));
  float cs[4], sn[4];
  Vec4<TA>::load(rope + (pos * 2) * kHeadDim + e0, cs);
  Vec4<TA>::load(rope + (pos * 2 + 1) * kHeadDim + e0, sn);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // rotate_half: element e pairs with e + 64 (lane j with lane j + 16)
    const float partner = __shfl_xor_sync(0xffffffffu, n[i], 16);
    const float rot = lane < 16 ? -partner : partner;
    out[i] = Act<TA>::round(Act<TA>::round(n[i] * cs[i]) + Act<TA>::round(rot * sn[i]));
  }
}

template <typename TA>
__global__ void __launch_bounds__(256) k8_qk_rope_kv(const TA *qkv, const TA *qn_w, const TA *kn_w, float eps,
                                                     const TA *rope, const int64_t *positions, int nh, int nkv,
                                                     int64_t max_len, TA *q_out, TA *k_cache, TA *v_cache,
                                                     uint32_t *status) {
  pdl_wait();
  const int t = blockIdx.x, lane = threadIdx.x & 31;
  const int hh = blockIdx.y * 8 + (threadIdx.x >> 5);
  const int nheads = nh + 2 * nkv;
  if (hh >= nheads) return;
  const int64_t pos = (int64_t)__ldcg(reinterpret_cast<const long long *>(positions) + t);
  if (pos < 0 || pos >= max_len) {
    if (lane == 0 && status) atomicOr(status, TM_STATUS_BAD_TOKEN_ID);
    return;
  }
  const int e0 = 4 * lane;
  float v[4];
  Vec4<TA>::load_cg(qkv + ((int64_t)t * nheads + hh) * kHeadDim + e0, v);
  pdl_trigger();
  if (hh >= nh + nkv) {  // v head: copy into the cache
    Vec4<TA>::store(v_cache + ((int64_t)(hh - nh - nkv) * max_len + pos) * kHeadDim + e0, v);
    return;
  }
  const bool is_q = hh < nh;
  float out[4];
  qk_norm_rope<TA>(v, is_q ? qn_w : kn_w, eps, rope, pos, lane, out);
  if (is_q)
    Vec4<TA>::store(q_out + ((int64_t)t * nh + hh) * kHeadDim + e0, out);
  else
    Vec4<TA>::store(k_cache + ((int64_t)(hh - nh) * max_len + pos) * kHeadDim + e0, out);
}

// ----------------------------------------------------- decode attention ----
// One query token, GQA: q head h reads KV head h / (nh / nkv).  Context =
// positions [0, pos] (pos from device memory, so a captured step replays at
// any position).  Grid (nkv, splits): CTA (g, s) takes the group's nh/nkv q
// heads (one warp each) over positions [s * chunk, min(n, (s + 1) * chunk))
// with chunk = ceil(n / splits) rounded up to 32.  K/V rows arrive 32 at a
// time by cp.async into a double-buffered shared tile.  Per tile a warp forms
// its 32 scores (lane j holds q[4j..4j+3]; the 32 partial dot products are
// summed across lanes by a 31-shuffle transposed reduction that leaves
// position i's score in lane i), then updates its running max, sum and
// output (fp32).  Each CTA writes (m, l, o[128]) per head; the last CTA of a
// KV head (counter in the workspace, reset by that CTA) merges the splits:
// out = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M), rounded to act.
template <typename TA>
__global__ void __launch_bounds__(kHeadMaxAttnWarps * 32) k8_attn_decode(
    const TA *q, const TA *k_cache, const TA *v_cache, const int64_t *position, int64_t max_len, int nh, int nkv,
    float scale, TA *out, float *part, unsigned *counters) {
  extern __shared__ __align__(16) uint8_t attn_smem[];
  TA *ks = reinterpret_cast<TA *>(attn_smem);                 // [2][32][128]
  TA *vs = ks + 2 * kAttnTile * kHeadDim;                     // [2][32][128]
  __shared__ unsigned s_last;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int G = nh / nkv;
  const int g = blockIdx.x, s = blockIdx.y, S = gridDim.y;
  const int h = g * G + w;
  pdl_wait();
  // context length; a position past the cache (refused by tm_qk_rope_kv) is clamped
  const int64_t n = min((int64_t)__ldcg(reinterpret_cast<const long long *>(position)) + 1, max_len);
  const int64_t per = ((n + S - 1) / S + kAttnTile - 1) / kAttnTile * kAttnTile;
  const int64_t p_begin = (int64_t)s * per;
  const int64_t p_end = min(n, p_begin + per);
  const TA *kbase = k_cache + (int64_t)g * max_len * kHeadDim;
  const TA *vbase = v_cache + (int64_t)g * max_len * kHeadDim;
  constexpr int kVecPerRow = kHeadDim * (int)sizeof(TA) / 16;

  auto issue = [&](int64_t p0, int buf) {
    const int rows = (int)min((int64_t)kAttnTile, p_end - p0);
    const int nvec = rows * kVecPerRow;
    for (int i = tid; i < nvec; i += blockDim.x) {
      const int r = i / kVecPerRow, c = i % kVecPerRow;
      const int64_t off = (p0 + r) * kHeadDim + c * (16 / (int)sizeof(TA));
      const int soff = (buf * kAttnTile + r) * kHeadDim + c * (16 / (int)sizeof(TA));
      cp_async16(ks + soff, kbase + off);
      cp_async16(vs + soff, vbase + off);
    }
    cp_async_commit();
  };

  float qv[4], o[4] = {0.f, 0.f, 0.f, 0.f};
  float m = -INFINITY, l = 0.f;
  Vec4<TA>::load_cg(q + (int64_t)h * kHeadDim + 4 * lane, qv);
  if (p_begin < p_end) issue(p_begin, 0);
  pdl_trigger();
  int buf = 0;
  for (int64_t p0 = p_begin; p0 < p_end; p0 += kAttnTile, buf ^= 1) {
    if (p0 + kAttnTile < p_end) {
      issue(p0 + kAttnTile, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int cnt = (int)min((int64_t)kAttnTile, p_end - p0);
    const TA *kt = ks + buf * kAttnTile * kHeadDim + 4 * lane;
    const TA *vt = vs + buf * kAttnTile * kHeadDim + 4 * lane;
    float sc[kAttnTile];
#pragma unroll
    for (int i = 0; i < kAttnTile; ++i) {
      float kk[4];
      Vec4<TA>::load(kt + i * kHeadDim, kk);
      sc[i] = qv[0] * kk[0];
#pragma unroll
      for (int e = 1; e < 4; ++e) sc[i] = fmaf(qv[e], kk[e], sc[i]);
    }
    // transposed reduction: afterwards sc[0] of lane i is position p0 + i's dot product
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
      const bool upper = (lane & off) != 0;
#pragma unroll
      for (int i = 0; i < off; ++i) {
        const float send = upper ? sc[i] : sc[i + off];
        const float keep = upper ? sc[i + off] : sc[i];
        sc[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
      }
    }
    const float my = lane < cnt ? sc[0] * scale : -INFINITY;
    const float m_new = fmaxf(m, warp_max(my));
    const float p = lane < cnt ? expf(my - m_new) : 0.f;
    const float corr = expf(m - m_new);   // 0 on the first tile (m = -inf)
    l = l * corr + warp_sum(p);
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] *= corr;
    for (int i = 0; i < cnt; ++i) {
      const float pi = __shfl_sync(0xffffffffu, p, i);
      float vv[4];
      Vec4<TA>::load(vt + i * kHeadDim, vv);
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = fmaf(pi, vv[e], o[e]);
    }
    m = m_new;
    __syncthreads();  // the next issue() overwrites this buffer
  }
  // partial of (head h, split s): m, l, o[128]
  float *pp = part + ((int64_t)h * S + s) * (kHeadDim + 4);
  if (lane == 0) {
    pp[0] = m;
    pp[1] = l;
  }
  *reinterpret_cast<float4 *>(pp + 4 + 4 * lane) = make_float4(o[0], o[1], o[2], o[3]);
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(counters + g, 1u) == (unsigned)(S - 1);
  __syncthreads();
  if (!s_last) return;
  if (tid == 0) counters[g] = 0u;  // self-resetting for the next call
  __threadfence();
  // merge: lane j holds the (m, l) of splits j, j + 32, ... (loads in flight
  // together), the weights e^(m_s - M) go to every lane by shuffles
  const float *ph = part + (int64_t)h * S * (kHeadDim + 4);
  float mj[2], lj[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int j = lane + 32 * u;
    const bool v = j < S;
    lj[u] = v ? __ldcg(ph + (int64_t)j * (kHeadDim + 4) + 1) : 0.f;
    mj[u] = v ? __ldcg(ph + (int64_t)j * (kHeadDim + 4)) : -INFINITY;
    if (!(lj[u] > 0.f)) mj[u] = -INFINITY;
  }
  const float M = warp_max(fmaxf(mj[0], mj[1]));
  float fj[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) fj[u] = lj[u] > 0.f ? expf(mj[u] - M) : 0.f;
  const float L = warp_sum(fj[0] * lj[0] + fj[1] * lj[1]);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j0 = 0; j0 < S; j0 += 8) {
    float4 oj[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      oj[u] = j0 + u < S ? __ldcg(reinterpret_cast<const float4 *>(ph + (int64_t)(j0 + u) * (kHeadDim + 4) + 4 + 4 * lane))
                         : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u;
      const float f = __shfl_sync(0xffffffffu, j < 32 ? fj[0] : fj[1], j & 31);
      if (j < S && f > 0.f) {
        acc[0] = fmaf(oj[u].x, f, acc[0]);
        acc[1] = fmaf(oj[u].y, f, acc[1]);
        acc[2] = fmaf(oj[u].z, f, acc[2]);
        acc[3] = fmaf(oj[u].w, f, acc[3]);
      }
    }
  }
  float res[4];
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) res[e] = acc[e] * inv;
  Vec4<TA>::store(out + (int64_t)h * kHeadDim + 4 * lane, res);
}

// ------------------------------------- decode attention on tensor cores ----
// 16-bit activations: the same split-K decode attention on mma.sync
// m16n8k16, the splits of one KV head in one thread-block cluster.  Grid
// (S, nkv), cluster (S, 1, 1), S <= 16: CTA (split s, KV head g) has 8 warps;
// warp w takes the 16-position tiles w, w + 8, ... of the split, each tile of
// K and V copied by the warp itself (cp.async, rows padded to 272 B:
// conflict-free ldmatrix; rows past the context zero-filled) into its own
// three-slot ring.  The products are transposed so that the group's G query
// heads are the MMA's N = 8 columns (NT = ceil(G / 8) column blocks) and the
// positions / head dims its M = 16 rows: S^T = K Q^T (A = K rows by ldmatrix,
// B = Q from registers), scaled, masked, online softmax per head (fp32, a
// column of S^T: shuffles across the 8 row lanes), then O^T += V^T P^T (A =
// V by ldmatrix.trans, B = P^T: the C fragment of S^T stored to shared
// memory as [position][head] and read back by ldmatrix.trans).  P is given
// as two 16-bit terms hi + lo so that the product carries P to about 2^-17
// relative like the fp32 reference (one 16-bit rounding of P alone moves
// outputs by more than an act-dtype ulp at short contexts).  Per 16 positions
// a warp issues 8 NT + 16 NT MMAs; two warps per SM sub-partition hide each
// other's MMA and shuffle latencies.  The warps' (m, l, O) merge through
// shared memory into the CTA's partial; after a cluster barrier each CTA
// reads every split's (m, l) and a slice of every split's O from distributed
// shared memory and writes that slice of
// out = sum_s O_s e^(m_s - M) / sum_s l_s e^(m_s - M).  No global
// workspace, fence or atomic: the merge costs one shared::cluster round trip
// instead of a device-scope release and a pass over L2.
constexpr int kAttnMmaWarps = 8;
constexpr int kMmaTile = 16;                          // positions per tile of a warp (one MMA row block)
constexpr int kMT = kMmaTile / 16;                    // MMA row blocks per tile
constexpr int kAttnMaxCluster = 16;
constexpr int kAttnRow = kHeadDim * 2 + 16;            // padded shared-memory row (bytes)
constexpr int kMmaTileBytes = kMmaTile * kAttnRow;    // one K or V tile
constexpr int kAttnStages = 3;                                    // tiles in flight per warp
constexpr int kAttnWarpBytes = kAttnStages * 2 * kMmaTileBytes;  // ring of K and V tiles
// shared memory: the warps' tile rings; each warp's P^T hi and lo [32][16 NT
// B].  After the loop the ring space holds each warp's O [warp][16][kAttnObRow]
// fp32 (row stride 132 floats: the scalar stores of a warp, heads 2t and dims
// g, hit 32 distinct banks) and the CTA's O [16][128] fp32.
constexpr int kAttnObRow = kHeadDim + 4;
constexpr int kAttnPOff = kAttnMmaWarps * kAttnWarpBytes;
constexpr int kAttnPWarpBytes = 2 * kMmaTile * 32;      // hi + lo, NT <= 2
constexpr int kAttnObufOff = 0;
constexpr int kAttnCtaOOff = kAttnObufOff + kAttnMmaWarps * 16 * kAttnObRow * 4;
constexpr int kAttnMmaSmem = kAttnPOff + kAttnMmaWarps * kAttnPWarpBytes;
static_assert(kAttnCtaOOff + 16 * kHeadDim * 4 <= kAttnPOff, "merge buffers fit in the tile rings");
static_assert(kAttnMmaSmem <= 227 * 1024, "k8_attn_mma shared memory");

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_cluster_f32x4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

template <typename TA> struct MmaOp;
template <> struct MmaOp<__half> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  // (a, b) as two 16-bit terms: hi = round(x), lo = round(x - hi)
  static __device__ __forceinline__ void split(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
  }
};
template <> struct MmaOp<__nv_bfloat16> {
  static __device__ __forceinline__ void run(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  static __device__ __forceinline__ void split(float a, float b, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(a - hf.x, b - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
  }
};
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Sequence b = blockIdx.z of a batch: its query q + b * nh * 128, its caches
// k_cache / v_cache + b * kv_bstride, its position position[b], its output
// out + b * nh * 128 (one sequence: gridDim.z = 1).
//
// kRope (one sequence): q points at the fused q/k/v projection output
// [(nh + 2 nkv) * 128] of this step instead of the rotated q; each CTA applies
// q_norm + rotary to its group's query heads itself (qk_norm_rope, the same
// arithmetic as k8_qk_rope_kv), and the CTA whose split holds this step's
// position applies k_norm + rotary to its KV head's k, appends k and v to the
// caches and puts them into its own tile (that row is not read from memory).
template <typename TA, int NT, bool kRope>
__global__ void __launch_bounds__(kAttnMmaWarps * 32) k8_attn_mma(const TA *q, const TA *k_cache, const TA *v_cache,
                                                                  const int64_t *position, int64_t max_len, int nh,
                                                                  int nkv, float scale, TA *out, int64_t kv_bstride,
                                                                  const TA *qn_w, const TA *kn_w, float eps,
                                                                  const TA *rope) {
  extern __shared__ __align__(128) uint8_t am_smem[];
  __shared__ float s_m[kAttnMmaWarps][16], s_l[kAttnMmaWarps][16];
  __shared__ float c_m[16], c_l[16];   // this CTA's partial (read by the cluster)
  __shared__ __align__(16) TA s_q[kRope ? 16 * kHeadDim : 8];     // kRope: the group's rotated q heads
  __shared__ __align__(16) TA s_kv[kRope ? 2 * kHeadDim : 8];     // kRope: this position's k and v
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int G = nh / nkv;
  const int s = (int)cluster_rank(), S = gridDim.x, gk = blockIdx.y;
  uint8_t *wbuf = am_smem + w * kAttnWarpBytes;
  const uint32_t p_hi = smem_u32(am_smem + kAttnPOff + w * kAttnPWarpBytes), p_lo = p_hi + kMmaTile * 16 * NT;
  float *obuf = reinterpret_cast<float *>(am_smem + kAttnObufOff);
  float *c_o = reinterpret_cast<float *>(am_smem + kAttnCtaOOff);
  const int64_t bz = blockIdx.z;
  q += bz * (kRope ? nh + 2 * nkv : nh) * kHeadDim;
  out += bz * nh * kHeadDim;
  pdl_wait();
  // context length; a position past the cache (refused by tm_qk_rope_kv) is clamped
  const int64_t n = min((int64_t)__ldcg(reinterpret_cast<const long long *>(position) + bz) + 1, max_len);
  const int64_t per = ((n + S - 1) / S + kMmaTile - 1) / kMmaTile * kMmaTile;
  const int64_t p_begin = (int64_t)s * per;
  const int64_t p_end = min(n, p_begin + per);
  const int ntiles = p_begin < p_end ? (int)((p_end - p_begin + kMmaTile - 1) / kMmaTile) : 0;
  const TA *kbase = k_cache + bz * kv_bstride + (int64_t)gk * max_len * kHeadDim;
  const TA *vbase = v_cache + bz * kv_bstride + (int64_t)gk * max_len * kHeadDim;
  // kRope: the position this step appends, when it falls in this split (a
  // position at or past the cache lies in no split: nothing is appended)
  const int64_t praw = kRope ? (int64_t)__ldcg(reinterpret_cast<const long long *>(position) + bz) : -1;
  const int64_t own_row = (kRope && praw >= p_begin && praw < p_end) ? praw : -1;
  // this warp's tiles: w, w + 4, ...; 32 rows x 16 pieces of 16 B of K and of V
  // (one cp.async group per tile slot, committed by the caller: empty groups
  // keep the count uniform, so the wait below is always "all but the newest
  // kAttnStages - 1")
  auto issue = [&](int ti, int buf) {
    const int64_t p0 = p_begin + (int64_t)ti * kMmaTile;
    const int cnt = (int)min((int64_t)kMmaTile, p_end - p0);
    const uint32_t kd = smem_u32(wbuf + buf * 2 * kMmaTileBytes), vd = kd + kMmaTileBytes;
#pragma unroll 4
    for (int i = lane; i < kMmaTile * 16; i += 32) {
      const int r = i >> 4, c = i & 15;
      const bool in = r < cnt && (!kRope || p0 + r != own_row);
      const int64_t off = (p0 + (in ? r : 0)) * kHeadDim + c * 8;
      cp_async16_z(kd + r * kAttnRow + c * 16, kbase + off, in ? 16 : 0);
      cp_async16_z(vd + r * kAttnRow + c * 16, vbase + off, in ? 16 : 0);
    }
  };
#pragma unroll
  for (int j = 0; j < kAttnStages - 1; ++j) {  // prologue: tiles w, w + 4, ...
    if (w + j * kAttnMmaWarps < ntiles) issue(w + j * kAttnMmaWarps, j);
    cp_async_commit();
  }
  if constexpr (kRope) {
    // the group's query heads: q_norm + rotary at this step's position
    const int64_t prope = min(max(praw, (int64_t)0), max_len - 1);
    for (int j = w; j < G; j += kAttnMmaWarps) {
      float v[4], r4[4];
      Vec4<TA>::load_cg(q + (int64_t)(gk * G + j) * kHeadDim + 4 * lane, v);
      qk_norm_rope<TA>(v, qn_w, eps, rope, prope, lane, r4);
      Vec4<TA>::store(s_q + j * kHeadDim + 4 * lane, r4);
    }
    if (own_row >= 0 && w == kAttnMmaWarps - 1) {  // this KV head's k (k_norm + rotary) and v
      float v[4], r4[4];
      Vec4<TA>::load_cg(q + (int64_t)(nh + gk) * kHeadDim + 4 * lane, v);
      qk_norm_rope<TA>(v, kn_w, eps, rope, own_row, lane, r4);
      Vec4<TA>::store(s_kv + 4 * lane, r4);
      Vec4<TA>::store(const_cast<TA *>(kbase) + own_row * kHeadDim + 4 * lane, r4);
      Vec4<TA>::load_cg(q + (int64_t)(nh + nkv + gk) * kHeadDim + 4 * lane, v);
      Vec4<TA>::store(s_kv + kHeadDim + 4 * lane, v);
      Vec4<TA>::store(const_cast<TA *>(vbase) + own_row * kHeadDim + 4 * lane, v);
    }
    __syncthreads();
  }
  // Q^T B fragments: column g8 of block nt = query head gk * G + 8 nt + g8 (zero past G);
  // k-step kk: dims 16 kk + 2 t4 (+1) and + 8
  uint32_t qb[NT][8][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int hh = nt * 8 + g8;
    if constexpr (kRope) {
      const TA *qh = s_q + (hh < G ? hh : 0) * kHeadDim;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[nt][kk][0] = hh < G ? *reinterpret_cast<const unsigned *>(qh + kk * 16 + 2 * t4) : 0u;
        qb[nt][kk][1] = hh < G ? *reinterpret_cast<const unsigned *>(qh + kk * 16 + 8 + 2 * t4) : 0u;
      }
    } else {
      const TA *qh = q + (int64_t)(gk * G + hh) * kHeadDim;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        qb[nt][kk][0] = hh < G ? __ldcg(reinterpret_cast<const unsigned *>(qh + kk * 16 + 2 * t4)) : 0u;
        qb[nt][kk][1] = hh < G ? __ldcg(reinterpret_cast<const unsigned *>(qh + kk * 16 + 8 + 2 * t4)) : 0u;
      }
    }
  }
  pdl_trigger();
  // O^T accumulators: block md = dims 16 md.., column block nt; element j:
  // dim 16 md + g8 (+8 for j >= 2), head 8 nt + 2 t4 + (j & 1)
  float o[8][NT][4];
#pragma unroll
  for (int md = 0; md < 8; ++md)
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) o[md][nt][0] = o[md][nt][1] = o[md][nt][2] = o[md][nt][3] = 0.f;
  float m_r[NT][2], l_r[NT][2];   // heads 8 nt + 2 t4 + e
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) m_r[nt][0] = m_r[nt][1] = -INFINITY, l_r[nt][0] = l_r[nt][1] = 0.f;
  int buf = 0;
  for (int ti = w; ti < ntiles; ti += kAttnMmaWarps, buf = buf == kAttnStages - 1 ? 0 : buf + 1) {
    {
      const int tn = ti + (kAttnStages - 1) * kAttnMmaWarps;
      if (tn < ntiles) issue(tn, buf == 0 ? kAttnStages - 1 : buf - 1);  // the slot tile ti - 4 used
      cp_async_commit();
      cp_async_wait<kAttnStages - 1>();
    }
    __syncwarp();
    if constexpr (kRope) {  // this step's k and v into their (zero-filled) row of the tile
      const int64_t p0 = p_begin + (int64_t)ti * kMmaTile;
      if (own_row >= p0 && own_row < p0 + kMmaTile) {
        const int r = (int)(own_row - p0), c = lane & 15;
        const uint4 val = *reinterpret_cast<const uint4 *>(s_kv + (lane < 16 ? 0 : kHeadDim) + c * 8);
        *reinterpret_cast<uint4 *>(wbuf + buf * 2 * kMmaTileBytes + (lane < 16 ? 0 : kMmaTileBytes) +
                                   r * kAttnRow + c * 16) = val;
        __syncwarp();
      }
    }
    const int cnt = (int)min((int64_t)kMmaTile, p_end - (p_begin + (int64_t)ti * kMmaTile));
    const uint32_t kd = smem_u32(wbuf + buf * 2 * kMmaTileBytes), vd = kd + kMmaTileBytes;
    // S^T = K Q^T: row blocks mt (positions 16 mt..) x column blocks nt, 8 steps of 16 dims
    float sc[kMT][NT][4];
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) sc[mt][nt][0] = sc[mt][nt][1] = sc[mt][nt][2] = sc[mt][nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      uint32_t a[kMT][4];
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt)  // matrices: rows +0/+8 x dims +0/+8
        ldsm_x4(kd + (mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * kAttnRow + (kk * 16 + (lane >> 4) * 8) * 2,
                a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) MmaOp<TA>::run(sc[mt][nt], a[mt], qb[nt][kk][0], qb[nt][kk][1]);
    }
    // scale, mask (position 16 mt + g8 + 8 (j >> 1) < cnt), running max per head
    float mx[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      mx[nt][0] = mx[nt][1] = -INFINITY;
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int pos = mt * 16 + g8 + (j >> 1) * 8;
          sc[mt][nt][j] = pos < cnt ? sc[mt][nt][j] * scale : -INFINITY;
          mx[nt][j & 1] = fmaxf(mx[nt][j & 1], sc[mt][nt][j]);
        }
    }
    float corr[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = mx[nt][e];
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 8));
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 16));
        const float mn = fmaxf(m_r[nt][e], v);
        corr[nt][e] = expf(m_r[nt][e] - mn);   // 0 on the first tile (m_r = -inf)
        m_r[nt][e] = mn;
      }
    float rs[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      rs[nt][0] = rs[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float v = sc[mt][nt][j];
          const float p = v == -INFINITY ? 0.f : expf(v - m_r[nt][j & 1]);
          sc[mt][nt][j] = p;
          rs[nt][j & 1] += p;
        }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float v = rs[nt][e];
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        v += __shfl_xor_sync(0xffffffffu, v, 8);
        v += __shfl_xor_sync(0xffffffffu, v, 16);
        l_r[nt][e] = l_r[nt][e] * corr[nt][e] + v;
      }
#pragma unroll
    for (int md = 0; md < 8; ++md)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) o[md][nt][j] *= corr[nt][j & 1];
    // P^T to shared memory, [position][head] as hi and lo 16-bit pairs
#pragma unroll
    for (int mt = 0; mt < kMT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t hi, lo;
          MmaOp<TA>::split(sc[mt][nt][2 * hf], sc[mt][nt][2 * hf + 1], hi, lo);
          const uint32_t off = (mt * 16 + g8 + 8 * hf) * (16 * NT) + nt * 16 + t4 * 4;
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(p_hi + off), "r"(hi) : "memory");
          asm volatile("st.shared.b32 [%0], %1;" ::"r"(p_lo + off), "r"(lo) : "memory");
        }
    __syncwarp();
    // B fragments of P^T (column block nt): one k-step of 16 positions per MMA row block
    uint32_t bh[NT][2 * kMT], bl[NT][2 * kMT];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if constexpr (kMT == 1) {  // matrices: hi positions 0-7, 8-15, lo positions 0-7, 8-15
        const uint32_t off = (lane & 15) * (16 * NT) + nt * 16;
        ldsm_x4_t((lane < 16 ? p_hi : p_lo) + off, bh[nt][0], bh[nt][1], bl[nt][0], bl[nt][1]);
      } else {  // matrices: positions 0-7, 8-15, 16-23, 24-31
        const uint32_t off = (lane & 31) * (16 * NT) + nt * 16;
        ldsm_x4_t(p_hi + off, bh[nt][0], bh[nt][1], bh[nt][2], bh[nt][3]);
        ldsm_x4_t(p_lo + off, bl[nt][0], bl[nt][1], bl[nt][2], bl[nt][3]);
      }
    }
    // O^T += V^T P^T: kMT steps of 16 positions x 8 row blocks of 16 dims
#pragma unroll
    for (int ks = 0; ks < kMT; ++ks) {
      uint32_t a[8][4];
      const int row = ks * 16 + (lane & 7) + ((lane >> 4) & 1) * 8;
#pragma unroll
      for (int md = 0; md < 8; ++md)  // transposed: dims +0/+8 x positions +0/+8
        ldsm_x4_t(vd + row * kAttnRow + (md * 16 + ((lane >> 3) & 1) * 8) * 2, a[md][0], a[md][1], a[md][2],
                  a[md][3]);
#pragma unroll
      for (int md = 0; md < 8; ++md)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) MmaOp<TA>::run(o[md][nt], a[md], bh[nt][2 * ks], bh[nt][2 * ks + 1]);
#pragma unroll
      for (int md = 0; md < 8; ++md)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) MmaOp<TA>::run(o[md][nt], a[md], bl[nt][2 * ks], bl[nt][2 * ks + 1]);
    }
    __syncwarp();  // the next issue() and P^T stores overwrite what this tile read
  }
  cp_async_wait<0>();
  __syncthreads();  // every warp is done with its tile ring, which now holds the merge buffers
  // ---- the CTA's partial: the warps' (m, l) and raw O, merged per head
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
    if (g8 == 0) {
      s_m[w][nt * 8 + 2 * t4] = m_r[nt][0];
      s_m[w][nt * 8 + 2 * t4 + 1] = m_r[nt][1];
      s_l[w][nt * 8 + 2 * t4] = l_r[nt][0];
      s_l[w][nt * 8 + 2 * t4 + 1] = l_r[nt][1];
    }
  {
    float *ob = obuf + w * 16 * kAttnObRow;
#pragma unroll
    for (int md = 0; md < 8; ++md)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int hh = nt * 8 + 2 * t4 + (j & 1);
          if (hh < G) ob[hh * kAttnObRow + md * 16 + g8 + (j >> 1) * 8] = o[md][nt][j];
        }
  }
  __syncthreads();
  for (int i = tid; i < G * kHeadDim / 4; i += kAttnMmaWarps * 32) {
    const int r = i / (kHeadDim / 4), c = 4 * (i % (kHeadDim / 4));
    float M = -INFINITY;
#pragma unroll
    for (int ww = 0; ww < kAttnMmaWarps; ++ww)
      if (s_l[ww][r] > 0.f) M = fmaxf(M, s_m[ww][r]);
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float L = 0.f;
#pragma unroll
    for (int ww = 0; ww < kAttnMmaWarps; ++ww) {
      const float f = s_l[ww][r] > 0.f ? expf(s_m[ww][r] - M) : 0.f;
      L += f * s_l[ww][r];
      const float4 v = *reinterpret_cast<const float4 *>(obuf + (ww * 16 + r) * kAttnObRow + c);
      acc.x = fmaf(v.x, f, acc.x);
      acc.y = fmaf(v.y, f, acc.y);
      acc.z = fmaf(v.z, f, acc.z);
      acc.w = fmaf(v.w, f, acc.w);
    }
    *reinterpret_cast<float4 *>(c_o + r * kHeadDim + c) = acc;
    if (c == 0) {
      c_m[r] = M;
      c_l[r] = L;
    }
  }
  cluster_sync_all();  // every split's partial is complete
  // ---- merge the splits through distributed shared memory: 4 lanes per
  // 4-dim output group (splits sub, sub + 4, ...); this CTA's groups are
  // s, s + S, ...  Every lane loads all it needs before using any of it.
  const int sub = lane & 3;
  for (int q0 = 0; q0 * S < G * kHeadDim / 4; q0 += kAttnMmaWarps * 8) {
    const int gi = s + S * (q0 + (tid >> 2));
    const bool valid = gi < G * kHeadDim / 4;
    const int r = valid ? gi / (kHeadDim / 4) : 0, c = valid ? 4 * (gi % (kHeadDim / 4)) : 0;
    float mj[kAttnMaxCluster / 4], lj[kAttnMaxCluster / 4];
    float4 oj[kAttnMaxCluster / 4];
#pragma unroll
    for (int u = 0; u < kAttnMaxCluster / 4; ++u) {
      const int j = sub + 4 * u;
      const bool in = valid && j < S;
      lj[u] = in ? ld_cluster_f32(cluster_addr(&c_l[r], j)) : 0.f;
      mj[u] = in ? ld_cluster_f32(cluster_addr(&c_m[r], j)) : -INFINITY;
      oj[u] = in ? ld_cluster_f32x4(cluster_addr(c_o + r * kHeadDim + c, j)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float M = -INFINITY;
#pragma unroll
    for (int u = 0; u < kAttnMaxCluster / 4; ++u)
      if (lj[u] > 0.f) M = fmaxf(M, mj[u]);
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 1));
    M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, 2));
    float L = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int u = 0; u < kAttnMaxCluster / 4; ++u) {
      const float f = lj[u] > 0.f ? expf(mj[u] - M) : 0.f;
      L = fmaf(f, lj[u], L);
      acc[0] = fmaf(oj[u].x, f, acc[0]);
      acc[1] = fmaf(oj[u].y, f, acc[1]);
      acc[2] = fmaf(oj[u].z, f, acc[2]);
      acc[3] = fmaf(oj[u].w, f, acc[3]);
    }
#pragma unroll
    for (int x = 1; x <= 2; x <<= 1) {
      L += __shfl_xor_sync(0xffffffffu, L, x);
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], x);
    }
    if (valid && sub == 0) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      float res[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) res[e] = acc[e] * inv;
      Vec4<TA>::store(out + (int64_t)(gk * G) * kHeadDim + 4 * gi, res);
    }
  }
  cluster_sync_all();  // the other CTAs have read this CTA's partial
}

// ------------------------------------------------- LM head + greedy argmax ----
// logits[r] = x . W[r] (W bf16 [vocab][hidden] as in the checkpoint, fp32
// accumulation, rounded to the act dtype for 16-bit activations), then the
// index of the largest logit, the lowest index among equal maxima (what
// torch.argmax returns), written to *token (int64).  A warp takes one row at
// a time (lane j: 16-byte chunks j, j + 32, ... of the row, x held in
// registers); per-CTA winners go to the workspace and the last CTA (counter,
// reset by that CTA) picks the overall one.
template <typename TX, int NCH>
__global__ void __launch_bounds__(256) k8_lm_head_argmax(const TX *x, const __nv_bfloat16 *w, int64_t vocab,
                                                         TX *logits, float *part_val, int64_t *part_idx,
                                                         unsigned *counter, int64_t *token) {
  constexpr int H = NCH * 256;
  __shared__ float s_val[8];
  __shared__ int64_t s_idx[8];
  __shared__ unsigned s_last;
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  float xr[NCH * 8];
  pdl_wait();
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int e = 0; e < 8; ++e) xr[c * 8 + e] = Act<TX>::to_f(Act<TX>::ld_cg(x + c * 256 + lane * 8 + e));
  pdl_trigger();
  float best = -INFINITY;
  int64_t best_i = INT64_MAX;
  const int64_t nw = (int64_t)gridDim.x * 8;
  for (int64_t r = (int64_t)blockIdx.x * 8 + wp; r < vocab; r += nw) {
    const __nv_bfloat16 *row = w + r * H + lane * 8;
    uint4 raw[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) raw[c] = ldg_stream(row + c * 256);
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const __nv_bfloat16 *b = reinterpret_cast<const __nv_bfloat16 *>(&raw[c]);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc = fmaf(xr[c * 8 + e], __bfloat162float(b[e]), acc);
    }
    acc = warp_sum(acc);
    const float lg = Act<TX>::round(acc);
    if (lane == 0 && logits) logits[r] = Act<TX>::from_f(lg);
    if (lg > best) {  // rows ascend within a warp: strict > keeps the lowest index
      best = lg;
      best_i = r;
    }
  }
  if (lane == 0) {
    s_val[wp] = best;
    s_idx[wp] = best_i;
  }
  __syncthreads();
  if (tid == 0) {
    float bv = s_val[0];
    int64_t bi = s_idx[0];
    for (int i = 1; i < 8; ++i)
      if (s_val[i] > bv || (s_val[i] == bv && s_idx[i] < bi)) {
        bv = s_val[i];
        bi = s_idx[i];
      }
    part_val[blockIdx.x] = bv;
    part_idx[blockIdx.x] = bi;
    __threadfence();
    s_last = atomicAdd(counter, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (!s_last) return;
  // last CTA: reduce the per-CTA winners
  __threadfence();
  float bv = -INFINITY;
  int64_t bi = INT64_MAX;
  for (int i = tid; i < (int)gridDim.x; i += 256) {
    const float v = __ldcg(part_val + i);
    const int64_t ix = (int64_t)__ldcg(reinterpret_cast<const long long *>(part_idx) + i);
    if (v > bv || (v == bv && ix < bi)) {
      bv = v;
      bi = ix;
    }
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int64_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    s_val[wp] = bv;
    s_idx[wp] = bi;
  }
  __syncthreads();
  if (tid == 0) {
    for (int i = 1; i < 8; ++i)
      if (s_val[i] > bv || (s_val[i] == bv && s_idx[i] < bi)) {
        bv = s_val[i];
        bi = s_idx[i];
      }
    *token = bi == INT64_MAX ? 0 : bi;
    *counter = 0u;
  }
}

constexpr int kLmHeadCTAs = 148 * 2;   // 2 CTAs of 256 threads per SM (96 registers a thread at hidden 2048)

}  // namespace tmoe

using namespace tmoe;

// ------------------------------------------------------------------ C ABI ----
namespace {
struct EmbedLaunch {
  const int64_t *ids; int64_t tokens; const void *table; int hidden; int64_t vocab; void *out; uint32_t *status;
  cudaStream_t s;
  template <typename TO> int run() {
    return launch_pdl(k8_embed<TO>, dim3((unsigned)tokens), dim3(256), 0, s, "k8_embed launch", ids,
                      (const __nv_bfloat16 *)table, hidden, vocab, (TO *)out, status);
  }
};
struct NormLaunch {
  const void *x; int64_t tokens; int hidden; const void *w; float eps; void *out; cudaStream_t s;
  template <typename TA> int run() {
    return launch_pdl(k8_rmsnorm<TA>, dim3((unsigned)tokens), dim3(256), 0, s, "k8_rmsnorm launch",
                      (const TA *)x, (const TA *)w, hidden, eps, (TA *)out);
  }
};
struct RopeLaunch {
  const void *qkv; int64_t tokens; int nh, nkv; const void *qn, *kn; float eps; const void *rope;
  const int64_t *pos; int64_t max_len; void *q_out, *k_cache, *v_cache; uint32_t *status; cudaStream_t s;
  template <typename TA> int run() {
    const dim3 grid((unsigned)tokens, (unsigned)((nh + 2 * nkv + 7) / 8));
    return launch_pdl(k8_qk_rope_kv<TA>, grid, dim3(256), 0, s, "k8_qk_rope_kv launch", (const TA *)qkv,
                      (const TA *)qn, (const TA *)kn, eps, (const TA *)rope, pos, nh, nkv, max_len, (TA *)q_out,
                      (TA *)k_cache, (TA *)v_cache, status);
  }
};
// Cluster size for k8_attn_mma: the requested splits (<= 16), halved until
// a cluster of that many CTAs (one SM each: the tiles take 136 KiB of shared
// memory) can be resident.  Sizes above 8 need the non-portable opt-in.
template <typename TA, int NT, bool kRope> int attn_mma_cluster(int *S) {
  static std::mutex mu;
  static int fits[kAttnMaxCluster + 1] = {};   // 0 unknown, 1 fits, -1 does not
  std::lock_guard<std::mutex> g(mu);
  int rc = ensure_smem(reinterpret_cast<const void *>(k8_attn_mma<TA, NT, kRope>), kAttnMmaSmem);
  if (rc) return rc;
  static bool opted = false;
  if (!opted) {
    rc = cuda_check(cudaFuncSetAttribute(k8_attn_mma<TA, NT, kRope>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1),
                    "cudaFuncSetAttribute(non-portable cluster)");
    if (rc) return rc;
    opted = true;
  }
  while (*S > 1) {
    if (fits[*S] == 0) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(*S, 1);
      cfg.blockDim = dim3(kAttnMmaWarps * 32);
      cfg.dynamicSmemBytes = kAttnMmaSmem;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = *S;
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      const cudaError_t e = cudaOccupancyMaxActiveClusters(&n, k8_attn_mma<TA, NT, kRope>, &cfg);
      if (e != cudaSuccess) {
        (void)cudaGetLastError();
        n = 0;
      }
      fits[*S] = n > 0 ? 1 : -1;
    }
    if (fits[*S] > 0) break;
    *S = *S / 2;
  }
  return TM_OK;
}

struct AttnLaunch {
  const void *q, *kc, *vc; const int64_t *pos; int64_t max_len; int nh, nkv, splits; float scale; void *out;
  float *part; unsigned *counters; cudaStream_t s;
  int batch = 1; int64_t kv_bstride = 0;
  const void *qn = nullptr, *kn = nullptr, *rope = nullptr; float eps = 0.f;   // q/k norm + rotary fused
  template <typename TA, int NT, bool kRope = false> int run_mma() {
    int S = std::min(splits, kAttnMaxCluster);
    int rc = attn_mma_cluster<TA, NT, kRope>(&S);
    if (rc) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S, nkv, batch);
    cfg.blockDim = dim3(kAttnMmaWarps * 32);
    cfg.dynamicSmemBytes = kAttnMmaSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cuda_check(cudaLaunchKernelEx(&cfg, k8_attn_mma<TA, NT, kRope>, (const TA *)q, (const TA *)kc,
                                         (const TA *)vc, pos, max_len, nh, nkv, scale, (TA *)out, kv_bstride,
                                         (const TA *)qn, (const TA *)kn, eps, (const TA *)rope),
                      "k8_attn_mma launch");
  }
  template <typename TA> int run() {
    if constexpr (sizeof(TA) == 2) {
      if (nh / nkv <= 8) return run_mma<TA, 1>();
      if (nh / nkv <= 16) return run_mma<TA, 2>();
    }
    const size_t smem = (size_t)4 * kAttnTile * kHeadDim * sizeof(TA);
    return launch_pdl(k8_attn_decode<TA>, dim3(nkv, splits), dim3(32 * (nh / nkv)), smem, s,
                      "k8_attn_decode launch", (const TA *)q, (const TA *)kc, (const TA *)vc, pos, max_len, nh,
                      nkv, scale, (TA *)out, part, counters);
  }
};
template <int NCH> struct LmHeadLaunch {
  const void *x; const void *w; int64_t vocab; void *logits; float *pv; int64_t *pi; unsigned *cnt;
  int64_t *token; cudaStream_t s;
  template <typename TX> int run() {
    return launch_pdl(k8_lm_head_argmax<TX, NCH>, dim3(kLmHeadCTAs), dim3(256), 0, s, "k8_lm_head_argmax launch",
                      (const TX *)x, (const __nv_bfloat16 *)w, vocab, (TX *)logits, pv, pi, cnt, token);
  }
};

int64_t attn_ws_bytes(int nh, int nkv, int splits) {
  return (int64_t)nh * splits * (kHeadDim + 4) * 4 + 256;
}
}  // namespace

extern "C" int tm_embed(const int64_t *ids, int64_t tokens, const void *table_bf16, int hidden, int64_t vocab,
                        int act_dtype, void *out, uint32_t *status, void *stream) {
  TM_REQUIRE(ids && table_bf16 && out, "null pointer");
  TM_REQUIRE(tokens >= 1 && tokens <= (1 << 20) && hidden > 0 && vocab > 0, "bad shape");
  EmbedLaunch f{ids, tokens, table_bf16, hidden, vocab, out, status, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_rmsnorm(const void *x, int64_t tokens, int hidden, int act_dtype, const void *weight, float eps,
                          void *out, void *stream) {
  TM_REQUIRE(x && weight && out, "null pointer");
  TM_REQUIRE(tokens >= 1 && tokens <= (1 << 20) && hidden > 0 && hidden % 4 == 0 && hidden <= 4096,
             "bad shape (hidden %d: a multiple of 4, at most 4096)", hidden);
  TM_REQUIRE(aligned(x, 16) && aligned(weight, 16) && aligned(out, 16), "buffers must be 16-byte aligned");
  NormLaunch f{x, tokens, hidden, weight, eps, out, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

extern "C" int tm_qk_rope_kv(const void *qkv, int64_t tokens, int n_heads, int n_kv_heads, int head_dim,
                             int act_dtype, const void *q_norm_w, const void *k_norm_w, float eps,
                             const void *rope_table, const int64_t *positions, int64_t max_len, void *q_out,
                             void *k_cache, void *v_cache, uint32_t *status, void *stream) {
  TM_REQUIRE(qkv && q_norm_w && k_norm_w && rope_table && positions && q_out && k_cache && v_cache,
             "null pointer");
  TM_REQUIRE(head_dim == kHeadDim, "head_dim %d unsupported (128)", head_dim);
  TM_REQUIRE(tokens >= 1 && tokens <= (1 << 20) && n_heads >= 1 && n_kv_heads >= 1 && max_len >= 1,
             "bad shape");
  TM_REQUIRE(aligned(qkv, 16) && aligned(q_out, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) &&
                 aligned(rope_table, 16),
             "buffers must be 16-byte aligned");
  RopeLaunch f{qkv, tokens, n_heads, n_kv_heads, q_norm_w, k_norm_w, eps, rope_table, positions, max_len,
               q_out, k_cache, v_cache, status, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

extern "C" int64_t tm_attn_decode_workspace_bytes(int n_heads, int n_kv_heads, int splits) {
  if (n_heads < 1 || n_kv_heads < 1 || splits < 1) return fail(TM_ERR_INVALID, "bad shape");
  return attn_ws_bytes(n_heads, n_kv_heads, splits);
}

extern "C" int tm_attn_decode(const void *q, const void *k_cache, const void *v_cache, const int64_t *position,
                              int64_t max_len, int n_heads, int n_kv_heads, int head_dim, int act_dtype,
                              float scale, int splits, void *out, void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(q && k_cache && v_cache && position && out && ws, "null pointer");
  TM_REQUIRE(head_dim == kHeadDim, "head_dim %d unsupported (128)", head_dim);
  TM_REQUIRE(n_kv_heads >= 1 && n_heads % n_kv_heads == 0 && n_heads / n_kv_heads <= kHeadMaxAttnWarps,
             "%d query heads over %d KV heads unsupported (at most %d per KV head)", n_heads, n_kv_heads,
             kHeadMaxAttnWarps);
  TM_REQUIRE(splits >= 1 && splits <= 64 && max_len >= 1, "bad splits %d (1..64) / max_len %lld", splits,
             (long long)max_len);
  TM_REQUIRE(aligned(q, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(out, 16) && aligned(ws, 16),
             "buffers must be 16-byte aligned");
  const int64_t need = attn_ws_bytes(n_heads, n_kv_heads, splits);
  if (ws_bytes < need) return fail(TM_ERR_WORKSPACE, "attention workspace %lld < %lld bytes", (long long)ws_bytes,
                                   (long long)need);
  float *part = static_cast<float *>(ws);
  unsigned *counters = reinterpret_cast<unsigned *>(static_cast<char *>(ws) + need - 256);
  TM_REQUIRE(n_kv_heads <= 64, "at most 64 KV heads");
  AttnLaunch f{q, k_cache, v_cache, position, max_len, n_heads, n_kv_heads, splits, scale, out, part, counters,
               as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

// A batch of sequences (batched decode): the same tensor-core kernel with the
// sequence as the grid's third dimension; 16-bit activations only.
struct AttnBatchLaunch {
  AttnLaunch f;
  template <typename TA> int run() {
    if constexpr (sizeof(TA) == 2) {
      if (f.nh / f.nkv <= 8) return f.run_mma<TA, 1>();
      return f.run_mma<TA, 2>();
    }
    return fail(TM_ERR_UNSUPPORTED, "batched decode attention needs 16-bit activations");
  }
};

extern "C" int tm_attn_decode_batched(const void *q, const void *k_cache, const void *v_cache,
                                      const int64_t *positions, int batch, int64_t kv_batch_stride,
                                      int64_t max_len, int n_heads, int n_kv_heads, int head_dim, int act_dtype,
                                      float scale, int splits, void *out, void *stream) {
  TM_REQUIRE(q && k_cache && v_cache && positions && out, "null pointer");
  TM_REQUIRE(head_dim == kHeadDim, "head_dim %d unsupported (128)", head_dim);
  TM_REQUIRE(act_dtype == TM_DTYPE_BF16 || act_dtype == TM_DTYPE_F16, "16-bit activations only");
  TM_REQUIRE(n_kv_heads >= 1 && n_kv_heads <= 65535 && n_heads % n_kv_heads == 0 && n_heads / n_kv_heads <= 16,
             "%d query heads over %d KV heads unsupported (at most 16 per KV head)", n_heads, n_kv_heads);
  TM_REQUIRE(batch >= 1 && batch <= 65535, "batch %d out of range (1..65535)", batch);
  TM_REQUIRE(splits >= 1 && max_len >= 1, "bad splits %d / max_len %lld", splits, (long long)max_len);
  TM_REQUIRE(kv_batch_stride >= (int64_t)n_kv_heads * max_len * kHeadDim || batch == 1,
             "kv_batch_stride %lld smaller than one sequence's cache", (long long)kv_batch_stride);
  TM_REQUIRE(kv_batch_stride % 8 == 0, "kv_batch_stride must keep rows 16-byte aligned");
  TM_REQUIRE(aligned(q, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(out, 16),
             "buffers must be 16-byte aligned");
  AttnBatchLaunch b{AttnLaunch{q, k_cache, v_cache, positions, max_len, n_heads, n_kv_heads, splits, scale, out,
                               nullptr, nullptr, as_stream(stream), batch, kv_batch_stride}};
  return dispatch_act(act_dtype, b);
}

// One step's q/k norm + rotary + KV append fused into the attention launch.
struct AttnRopeLaunch {
  AttnLaunch f;
  template <typename TA> int run() {
    if constexpr (sizeof(TA) == 2) {
      if (f.nh / f.nkv <= 8) return f.run_mma<TA, 1, true>();
      return f.run_mma<TA, 2, true>();
    }
    return fail(TM_ERR_UNSUPPORTED, "the fused q/k rotary + attention needs 16-bit activations");
  }
};

extern "C" int tm_qk_rope_attn_decode(const void *qkv, const void *q_norm_w, const void *k_norm_w, float eps,
                                      const void *rope_table, const int64_t *position, int64_t max_len, int n_heads,
                                      int n_kv_heads, int head_dim, int act_dtype, float scale, int splits,
                                      void *k_cache, void *v_cache, void *out, void *stream) {
  TM_REQUIRE(qkv && q_norm_w && k_norm_w && rope_table && position && k_cache && v_cache && out, "null pointer");
  TM_REQUIRE(head_dim == kHeadDim, "head_dim %d unsupported (128)", head_dim);
  TM_REQUIRE(act_dtype == TM_DTYPE_BF16 || act_dtype == TM_DTYPE_F16, "16-bit activations only");
  TM_REQUIRE(n_kv_heads >= 1 && n_kv_heads <= 65535 && n_heads % n_kv_heads == 0 && n_heads / n_kv_heads <= 16,
             "%d query heads over %d KV heads unsupported (at most 16 per KV head)", n_heads, n_kv_heads);
  TM_REQUIRE(splits >= 1 && max_len >= 1, "bad splits %d / max_len %lld", splits, (long long)max_len);
  TM_REQUIRE(aligned(qkv, 16) && aligned(k_cache, 16) && aligned(v_cache, 16) && aligned(out, 16) &&
                 aligned(rope_table, 16),
             "buffers must be 16-byte aligned");
  AttnRopeLaunch b{AttnLaunch{qkv, k_cache, v_cache, position, max_len, n_heads, n_kv_heads, splits, scale, out,
                              nullptr, nullptr, as_stream(stream), 1, 0, q_norm_w, k_norm_w, rope_table, eps}};
  return dispatch_act(act_dtype, b);
}

extern "C" int64_t tm_lm_head_workspace_bytes(void) {
  return (int64_t)kLmHeadCTAs * (4 + 8) + 256;
}

extern "C" int tm_lm_head_argmax(const void *x, int hidden, int act_dtype, const void *w_bf16, int64_t vocab,
                                 void *logits, int64_t *token, void *ws, int64_t ws_bytes, void *stream) {
  TM_REQUIRE(x && w_bf16 && token && ws, "null pointer");
  TM_REQUIRE(vocab >= 1 && hidden % 256 == 0 && hidden >= 256 && hidden <= 4096,
             "hidden %d must be a multiple of 256 in [256, 4096]", hidden);
  TM_REQUIRE(aligned(w_bf16, 16) && aligned(x, 16) && aligned(ws, 16), "buffers must be 16-byte aligned");
  if (ws_bytes < tm_lm_head_workspace_bytes())
    return fail(TM_ERR_WORKSPACE, "LM-head workspace %lld < %lld bytes", (long long)ws_bytes,
                (long long)tm_lm_head_workspace_bytes());
  char *b = static_cast<char *>(ws);
  int64_t *pi = reinterpret_cast<int64_t *>(b);
  float *pv = reinterpret_cast<float *>(b + (int64_t)kLmHeadCTAs * 8);
  unsigned *cnt = reinterpret_cast<unsigned *>(b + (int64_t)kLmHeadCTAs * 12 + 128 - ((int64_t)kLmHeadCTAs * 12) % 128);
  cudaStream_t s = as_stream(stream);
  switch (hidden / 256) {
#define TM_LMH(N)                                                                   \
  case N: {                                                                          \
    LmHeadLaunch<N> f{x, w_bf16, vocab, logits, pv, pi, cnt, token, s};              \
    return dispatch_act(act_dtype, f);                                               \
  }
    TM_LMH(1) TM_LMH(2) TM_LMH(4) TM_LMH(8) TM_LMH(16)
#undef TM_LMH
    default: return fail(TM_ERR_UNSUPPORTED, "hidden %d unsupported (256 * {1, 2, 4, 8, 16})", hidden);
  }
}

// Qwen3.5 linear attention (gated delta rule), one decode step in one launch.
//
// The reference runs Hugging Face's Qwen3_5MoeGatedDeltaNet for the 30 of 40
// Qwen3.5 layers whose layer type is "linear_attention"
// (execution/layer_executor.py:134-139; its per-layer conv and recurrent
// states live in cache/qwen35_cache.py:43-64).  Without the optional fused
// libraries that module runs, per decode token (transformers 5.5.0,
// models/qwen3_5_moe/modeling_qwen3_5_moe.py):
//   torch_causal_conv1d_update (:211-226): shift the K-column conv state left,
//     append this token's in_proj_qkv row, depthwise conv over the K columns,
//     SiLU, rounded to the act dtype;
//   :495-507: beta = sigmoid(b), g = -exp(A_log) * softplus(a + dt_bias);
//   torch_recurrent_gated_delta_rule (:315-354) with use_qk_l2norm_in_kernel:
//     l2norm(q), l2norm(k) in the act dtype, q /= sqrt(d_k); per value head,
//     S = S * exp(g); kv = S^T k; delta = (v - kv) * beta; S += k delta^T;
//     o = S^T q (fp32 state);
//   Qwen3_5MoeRMSNormGated (:176-191): RMSNorm of o over the head, weight,
//     times silu(z).
// This kernel does all of it for one (sequence, value head) per CTA; the
// in/out projections stay plain GEMMs of the caller.
//
// Layout (row-major, contiguous):
//   qkv        [B][2*Hk*128 + Hv*128]  q heads, k heads, v heads (torch.split order)
//   z          [B][Hv*128]; a, b [B][Hv]
//   conv_w     [conv_dim][K]           conv1d.weight without its middle axis
//   conv_in    [B][conv_dim][K]        read only; conv_out the shifted state
//   state      [B][Hv][128][128] fp32  S[d_k][d_v], updated in place
//   out        [B][Hv*128]             gated-normed output (in front of out_proj)
// A CTA of 512 threads owns the whole 64 KB state of its head: warp w holds
// state rows 8w..8w+7, lane l columns 4l..4l+3 (one 16-byte load per row), so
// the state is read and written once, coalesced, and never leaves registers
// between the decay, the two contractions and the rank-1 update.  The state
// (4 MB per layer of Qwen3.5 at batch 1) is the algorithmic traffic: the
// kernel is HBM-bound.
#include "tm_common.cuh"

namespace tmoe {
namespace {

constexpr int kGdnDim = 128;                    // key and value head dim
constexpr int kGdnThreads = 512;
constexpr int kGdnWarps = kGdnThreads / 32;      // 16
constexpr int kGdnRows = kGdnDim / kGdnWarps;    // 8 state rows per warp
constexpr int kGdnMaxConv = 8;                   // conv kernel sizes 1..8

__device__ __forceinline__ float gdn_silu(float x) { return x / (1.f + expf(-x)); }

template <typename TA>
__global__ void __launch_bounds__(kGdnThreads) k9_gdn_decode(
    const TA *qkv, const TA *z, const TA *a_in, const TA *b_in, const TA *conv_w, const float *A_log,
    const float *dt_bias, const TA *norm_w, const TA *conv_in, TA *conv_out, float *state, TA *out,
    int n_k_heads, int n_v_heads, int K, float q_scale, float eps) {
  __shared__ float s_q[kGdnDim], s_k[kGdnDim], s_v[kGdnDim], s_delta[kGdnDim];
  __shared__ float s_red[kGdnWarps][kGdnDim];
  __shared__ float s_l2[8];      // per-warp sums of squares: q in warps 0-3, k in warps 4-7
  __shared__ float s_nrm[4];     // per-warp sums of squares of o
  __shared__ float s_gate[2];    // beta, exp(g)

  const int h = blockIdx.x, bt = blockIdx.y;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int ratio = n_v_heads / n_k_heads, kh = h / ratio;
  const int key_dim = n_k_heads * kGdnDim;
  const int conv_dim = 2 * key_dim + n_v_heads * kGdnDim;

  // Conv channel of this thread: q (threads 0-127) and k (128-255) of key
  // head kh (repeat_interleave: value head h reads key head h / ratio), v of
  // value head h (256-383); threads 384-511 have none.
  int ch = -1;
  if (tid < 128) ch = kh * kGdnDim + tid;
  else if (tid < 256) ch = key_dim + kh * kGdnDim + (tid - 128);
  else if (tid < 384) ch = 2 * key_dim + h * kGdnDim + (tid - 256);

  // Weights (written by no kernel of the step) before the dependency wait.
  float wc[kGdnMaxConv];
#pragma unroll
  for (int j = 0; j < kGdnMaxConv; ++j)
    wc[j] = (ch >= 0 && j < K) ? Act<TA>::to_f(conv_w[(int64_t)ch * K + j]) : 0.f;
  const float nw = tid < kGdnDim ? Act<TA>::to_f(norm_w[tid]) : 0.f;
  float a_log = 0.f, dtb = 0.f;
  if (tid == 384) {
    a_log = A_log[h];
    dtb = dt_bias[h];
  }

  pdl_wait();

  // The head's state: issued first, consumed after the conv and the norms.
  float *S = state + ((int64_t)bt * n_v_heads + h) * (kGdnDim * kGdnDim);
  float s[kGdnRows][4];
#pragma unroll
  for (int r = 0; r < kGdnRows; ++r) {
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(S + (w * kGdnRows + r) * kGdnDim + 4 * lane));
    s[r][0] = v.x; s[r][1] = v.y; s[r][2] = v.z; s[r][3] = v.w;
  }
  pdl_trigger();

  // Causal conv update of this thread's channel (torch_causal_conv1d_update).
  float y = 0.f;
  if (ch >= 0) {
    const int64_t row = (int64_t)bt * conv_dim + ch;
    const TA *ci = conv_in + row * K;
    float nv[kGdnMaxConv];
#pragma unroll
    for (int j = 0; j < kGdnMaxConv; ++j)
      if (j < K - 1) nv[j] = Act<TA>::to_f(Act<TA>::ld_cg(ci + j + 1));
    const float x = Act<TA>::to_f(Act<TA>::ld_cg(qkv + row));
#pragma unroll
    for (int j = 0; j < kGdnMaxConv; ++j)
      if (j == K - 1) nv[j] = x;
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < kGdnMaxConv; ++j)
      if (j < K) acc = fmaf(nv[j], wc[j], acc);
    y = Act<TA>::round(gdn_silu(Act<TA>::round(acc)));
    // q/k channels are shared by the `ratio` value heads of key head kh: the
    // first of them writes their new state; every CTA reads conv_in only.
    if (tid >= 256 || h % ratio == 0) {
      TA *co = conv_out + row * K;
#pragma unroll
      for (int j = 0; j < kGdnMaxConv; ++j)
        if (j < K) co[j] = Act<TA>::from_f(nv[j]);
    }
  }
  // l2norm in the act dtype: round(x*x), fp32 sum rounded, + 1e-6, rsqrt.
  if (tid < 256) {
    const float sq = warp_sum(Act<TA>::round(y * y));
    if (lane == 0) s_l2[w] = sq;
  } else if (tid < 384) {
    s_v[tid - 256] = y;
  } else if (tid == 384) {
    const float bv = Act<TA>::to_f(Act<TA>::ld_cg(b_in + (int64_t)bt * n_v_heads + h));
    const float av = Act<TA>::to_f(Act<TA>::ld_cg(a_in + (int64_t)bt * n_v_heads + h));
    const float xa = av + dtb;
    const float sp = xa > 20.f ? xa : log1pf(expf(xa));   // softplus, threshold 20
    const float g = __fmul_rn(-expf(a_log), sp);
    s_gate[0] = Act<TA>::round(1.f / (1.f + expf(-bv)));  // sigmoid in the act dtype
    s_gate[1] = expf(g);
  }
  __syncthreads();
  if (tid < 256) {
    const int base = tid < 128 ? 0 : 4;
    float ss = Act<TA>::round(((s_l2[base] + s_l2[base + 1]) + s_l2[base + 2]) + s_l2[base + 3]);
    ss = Act<TA>::round(ss + 1e-6f);
    const float inv = Act<TA>::round(rsqrtf(ss));
    const float yn = Act<TA>::round(y * inv);
    if (tid < 128) s_q[tid] = __fmul_rn(yn, q_scale);
    else s_k[tid - 128] = yn;
  }
  __syncthreads();

  // Recurrence (fp32, the reference's separate roundings of each product).
  const float beta = s_gate[0], decay = s_gate[1];
  float kr[kGdnRows], qr[kGdnRows];
#pragma unroll
  for (int r = 0; r < kGdnRows; ++r) {
    kr[r] = s_k[w * kGdnRows + r];
    qr[r] = s_q[w * kGdnRows + r];
  }
  float p[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int r = 0; r < kGdnRows; ++r)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      s[r][e] = __fmul_rn(s[r][e], decay);
      p[e] = __fadd_rn(p[e], __fmul_rn(s[r][e], kr[r]));
    }
#pragma unroll
  for (int e = 0; e < 4; ++e) s_red[w][4 * lane + e] = p[e];
  __syncthreads();
  if (tid < kGdnDim) {
    float kv = 0.f;
#pragma unroll
    for (int i = 0; i < kGdnWarps; ++i) kv = __fadd_rn(kv, s_red[i][tid]);
    s_delta[tid] = __fmul_rn(__fsub_rn(s_v[tid], kv), beta);
  }
  __syncthreads();
  float d[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    d[e] = s_delta[4 * lane + e];
    p[e] = 0.f;
  }
#pragma unroll
  for (int r = 0; r < kGdnRows; ++r) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      s[r][e] = __fadd_rn(s[r][e], __fmul_rn(kr[r], d[e]));
      p[e] = __fadd_rn(p[e], __fmul_rn(s[r][e], qr[r]));
    }
    *reinterpret_cast<float4 *>(S + (w * kGdnRows + r) * kGdnDim + 4 * lane) =
        make_float4(s[r][0], s[r][1], s[r][2], s[r][3]);
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) s_red[w][4 * lane + e] = p[e];
  __syncthreads();

  // Gated RMSNorm over the head (Qwen3_5MoeRMSNormGated, norm before gate).
  float oa = 0.f;
  if (tid < kGdnDim) {
    float o = 0.f;
#pragma unroll
    for (int i = 0; i < kGdnWarps; ++i) o = __fadd_rn(o, s_red[i][tid]);
    oa = Act<TA>::round(o);
    const float sq = warp_sum(__fmul_rn(oa, oa));
    if (lane == 0) s_nrm[w] = sq;
  }
  __syncthreads();
  if (tid < kGdnDim) {
    const float var = (((s_nrm[0] + s_nrm[1]) + s_nrm[2]) + s_nrm[3]) / (float)kGdnDim;
    const float hn = Act<TA>::round(oa * rsqrtf(var + eps));
    const float wn = Act<TA>::round(nw * hn);
    const int64_t oi = ((int64_t)bt * n_v_heads + h) * kGdnDim + tid;
    const float zf = Act<TA>::to_f(Act<TA>::ld_cg(z + oi));
    out[oi] = Act<TA>::from_f(wn * gdn_silu(zf));
  }
}

struct GdnLaunch {
  const void *qkv, *z, *a, *b, *conv_w; const float *A_log, *dt_bias; const void *norm_w; float eps;
  const void *conv_in; void *conv_out; float *state; void *out; int64_t batch; int hk, hv, K; cudaStream_t s;
  template <typename TA> int run() {
    const float q_scale = (float)(1.0 / sqrt((double)kGdnDim));
    return launch_pdl(k9_gdn_decode<TA>, dim3((unsigned)hv, (unsigned)batch), dim3(kGdnThreads), 0, s,
                      "k9_gdn_decode launch", (const TA *)qkv, (const TA *)z, (const TA *)a, (const TA *)b,
                      (const TA *)conv_w, A_log, dt_bias, (const TA *)norm_w, (const TA *)conv_in,
                      (TA *)conv_out, state, (TA *)out, hk, hv, K, q_scale, eps);
  }
};

bool overlap(const void *p, int64_t pn, const void *q, int64_t qn) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p), b = reinterpret_cast<uintptr_t>(q);
  return a < b + (uintptr_t)qn && b < a + (uintptr_t)pn;
}

}  // namespace
}  // namespace tmoe

using namespace tmoe;

extern "C" int tm_gdn_decode(const void *qkv, const void *z, const void *a, const void *b, int64_t batch,
                             int n_k_heads, int n_v_heads, int head_k_dim, int head_v_dim, int conv_kernel,
                             int act_dtype, const void *conv_w, const float *A_log, const float *dt_bias,
                             const void *norm_w, float eps, const void *conv_state_in, void *conv_state_out,
                             float *recurrent_state, void *out, void *stream) {
  TM_REQUIRE(qkv && z && a && b && conv_w && A_log && dt_bias && norm_w && conv_state_in && conv_state_out &&
                 recurrent_state && out,
             "null pointer");
  TM_REQUIRE(head_k_dim == kGdnDim && head_v_dim == kGdnDim, "head dims %d/%d unsupported (128/128)", head_k_dim,
             head_v_dim);
  TM_REQUIRE(batch >= 1 && batch <= 65535, "batch %lld outside [1, 65535]", (long long)batch);
  TM_REQUIRE(n_k_heads >= 1 && n_v_heads >= n_k_heads && n_v_heads % n_k_heads == 0 && n_v_heads <= 4096,
             "%d value heads over %d key heads unsupported (a multiple, at most 4096)", n_v_heads, n_k_heads);
  TM_REQUIRE(conv_kernel >= 1 && conv_kernel <= kGdnMaxConv, "conv kernel %d outside [1, %d]", conv_kernel,
             kGdnMaxConv);
  TM_REQUIRE(act_dtype == TM_DTYPE_F32 || act_dtype == TM_DTYPE_F16 || act_dtype == TM_DTYPE_BF16,
             "unknown act dtype %d", act_dtype);
  const int64_t esz = act_dtype == TM_DTYPE_F32 ? 4 : 2;
  TM_REQUIRE(aligned(recurrent_state, 16), "recurrent_state must be 16-byte aligned");
  TM_REQUIRE(aligned(qkv, esz) && aligned(z, esz) && aligned(a, esz) && aligned(b, esz) && aligned(conv_w, esz) &&
                 aligned(norm_w, esz) && aligned(conv_state_in, esz) && aligned(conv_state_out, esz) &&
                 aligned(out, esz) && aligned(A_log, 4) && aligned(dt_bias, 4),
             "buffers must be aligned to their element size");
  const int64_t conv_dim = 2LL * n_k_heads * kGdnDim + (int64_t)n_v_heads * kGdnDim;
  const int64_t conv_bytes = batch * conv_dim * conv_kernel * esz;
  TM_REQUIRE(!overlap(conv_state_in, conv_bytes, conv_state_out, conv_bytes),
             "conv_state_in and conv_state_out must not overlap (value heads sharing a key head read the old "
             "state while one of them writes the new one)");
  GdnLaunch f{qkv, z, a, b, conv_w, A_log, dt_bias, norm_w, eps, conv_state_in, conv_state_out, recurrent_state,
              out, batch, n_k_heads, n_v_heads, conv_kernel, as_stream(stream)};
  return dispatch_act(act_dtype, f);
}

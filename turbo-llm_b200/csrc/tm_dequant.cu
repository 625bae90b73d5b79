// K0 (FP8 block dequantisation) and K5 (packed expert layout: pack / unpack).
#include "tm_common.cuh"

namespace tmoe {

// out = cast(w) * cast(scale), evaluated as the reference does in the output
// dtype (loader/expert_loader.py:153-160): both operands are converted to the
// output dtype, multiplied in fp32 and rounded once.  e4m3 -> f16/bf16/f32 is
// exact, so only the scale conversion and the product round.
template <typename TO> struct DQ;
template <> struct DQ<float> {
  static __device__ __forceinline__ float prep_scale(float s) { return s; }
  static __device__ __forceinline__ float make(float w, float s) { return __fmul_rn(w, s); }
};
template <> struct DQ<__half> {
  static __device__ __forceinline__ float prep_scale(float s) { return __half2float(__float2half_rn(s)); }
  static __device__ __forceinline__ __half make(float w, float s) { return __float2half_rn(__fmul_rn(w, s)); }
};
template <> struct DQ<__nv_bfloat16> {
  static __device__ __forceinline__ float prep_scale(float s) {
    return __bfloat162float(__float2bfloat16_rn(s));
  }
  static __device__ __forceinline__ __nv_bfloat16 make(float w, float s) {
    return __float2bfloat16_rn(__fmul_rn(w, s));
  }
};

// Dequantise 16 consecutive e4m3 values (one 16-byte chunk) with one scale.
template <typename TO>
__device__ __forceinline__ void dq16(uint4 v, float s, TO *dst) {
  const float sc = DQ<TO>::prep_scale(s);
  uint32_t w[4] = {v.x, v.y, v.z, v.w};
  TO o[16];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float a, b, c, d;
    e4m3x4_to_f32(w[i], a, b, c, d);
    o[4 * i + 0] = DQ<TO>::make(a, sc);
    o[4 * i + 1] = DQ<TO>::make(b, sc);
    o[4 * i + 2] = DQ<TO>::make(c, sc);
    o[4 * i + 3] = DQ<TO>::make(d, sc);
  }
  // 16 * sizeof(TO) bytes: 32 (f16/bf16) or 64 (f32), written as 16-byte vectors
  const uint4 *src = reinterpret_cast<const uint4 *>(o);
  uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
  for (int i = 0; i < (int)(16 * sizeof(TO) / 16); ++i) d4[i] = src[i];
}

template <typename TO>
__global__ void k0_dequant(const uint8_t *__restrict__ w, const float *__restrict__ s, int64_t rows,
                           int64_t cols, TO *__restrict__ out) {
  const int64_t chunks_per_row = cols / 16;
  const int64_t n = rows * chunks_per_row;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / chunks_per_row;
    const int64_t c = (i % chunks_per_row) * 16;
    const uint4 v = *reinterpret_cast<const uint4 *>(w + r * cols + c);
    const float sc = s[(r / 128) * (cols / 128) + c / 128];
    dq16<TO>(v, sc, out + r * cols + c);
  }
}

// ---------------------------------------------------------------- pack ----
// w13 unit u (16 bytes) -> (e, rg, kc, mat, r); row = rg*kRows+r, col = kc*16
__global__ void k5_pack_w13(const uint8_t *__restrict__ gate, const uint8_t *__restrict__ up,
                            int n, int H, int I, uint8_t *__restrict__ w13) {
  const int KC = H / 16, RG = I / kRows;
  const int64_t units = (int64_t)n * RG * KC * 2 * kRows;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = u;
    const int lane = t % kRows; t /= kRows;
    const int mat = t % 2; t /= 2;
    const int kc = t % KC; t /= KC;
    const int rg = t % RG; t /= RG;
    const int64_t e = t;
    const int64_t r = rg * kRows + lane;
    const uint8_t *src = (mat ? up : gate) + (e * I + r) * H + (int64_t)kc * 16;
    reinterpret_cast<uint4 *>(w13)[u] = *reinterpret_cast<const uint4 *>(src);
  }
}

__global__ void k5_pack_s13(const float *__restrict__ gs, const float *__restrict__ us, int n,
                            int H, int I, float *__restrict__ s13) {
  const int HB = H / 128, IB = I / 128;
  const int64_t total = (int64_t)n * IB * 2 * HB;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = i;
    const int hb = t % HB; t /= HB;
    const int mat = t % 2; t /= 2;
    const int ib = t % IB; t /= IB;
    const int64_t e = t;
    s13[i] = (mat ? us : gs)[(e * IB + ib) * HB + hb];
  }
}

// w2 unit u -> (e, rgo, kc, r); row = rgo*kRows+r (0..H), col = kc*16 (0..I)
__global__ void k5_pack_w2(const uint8_t *__restrict__ down, int n, int H, int I,
                           uint8_t *__restrict__ w2) {
  const int KC = I / 16, RG = H / kRows;
  const int64_t units = (int64_t)n * RG * KC * kRows;
  for (int64_t u = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; u < units;
       u += (int64_t)gridDim.x * blockDim.x) {
    int64_t t = u;
    const int lane = t % kRows; t /= kRows;
    const int kc = t % KC; t /= KC;
    const int rg = t % RG; t /= RG;
    const int64_t e = t;
    const int64_t r = rg * kRows + lane;
    const uint8_t *src = down + (e * H + r) * I + (int64_t)kc * 16;
    reinterpret_cast<uint4 *>(w2)[u] = *reinterpret_cast<const uint4 *>(src);
  }
}

// Dense dequantised gate/up ([I,H]) from the packed w13 of one expert.
template <typename TO>
__global__ void k5_unpack_w13(const uint8_t *__restrict__ w13, const float *__restrict__ s13, int H,
                              int I, int mat, TO *__restrict__ out) {
  const int KC = H / 16, HB = H / 128;
  const int64_t n = (int64_t)I * KC;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = i / KC, kc = i % KC;
    const int64_t u = (((int64_t)(r / kRows) * KC + kc) * 2 + mat) * kRows + (r % kRows);
    const uint4 v = reinterpret_cast<const uint4 *>(w13)[u];
    const float sc = s13[((r / 128) * 2 + mat) * HB + (kc * 16) / 128];
    dq16<TO>(v, sc, out + (int64_t)r * H + kc * 16);
  }
}

template <typename TO>
__global__ void k5_unpack_w2(const uint8_t *__restrict__ w2, const float *__restrict__ s2, int H,
                             int I, TO *__restrict__ out) {
  const int KC = I / 16, IB = I / 128;
  const int64_t n = (int64_t)H * KC;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = i / KC, kc = i % KC;
    const int64_t u = ((int64_t)(r / kRows) * KC + kc) * kRows + (r % kRows);
    const uint4 v = reinterpret_cast<const uint4 *>(w2)[u];
    const float sc = s2[(r / 128) * IB + (kc * 16) / 128];
    dq16<TO>(v, sc, out + (int64_t)r * I + kc * 16);
  }
}

static int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  if (g > 148 * 64) g = 148 * 64;
  return g < 1 ? 1 : static_cast<int>(g);
}

}  // namespace tmoe

using namespace tmoe;

extern "C" int tm_dequant_fp8_block(const uint8_t *w, const float *scale_inv, int64_t rows,
                                    int64_t cols, void *out, int out_dtype, void *stream) {
  TM_REQUIRE(w && scale_inv && out, "null pointer");
  TM_REQUIRE(rows > 0 && cols > 0 && rows % 128 == 0 && cols % 128 == 0,
             "rows (%lld) and cols (%lld) must be positive multiples of 128", (long long)rows,
             (long long)cols);
  TM_REQUIRE(aligned(w, 16) && aligned(out, 16), "w and out must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const int threads = 256;
  const int grid = grid_for(rows * cols / 16, threads);
  switch (out_dtype) {
    case TM_DTYPE_F32: k0_dequant<float><<<grid, threads, 0, s>>>(w, scale_inv, rows, cols, (float *)out); break;
    case TM_DTYPE_F16: k0_dequant<__half><<<grid, threads, 0, s>>>(w, scale_inv, rows, cols, (__half *)out); break;
    case TM_DTYPE_BF16:
      k0_dequant<__nv_bfloat16><<<grid, threads, 0, s>>>(w, scale_inv, rows, cols, (__nv_bfloat16 *)out);
      break;
    default: return fail(TM_ERR_INVALID, "unknown out dtype %d", out_dtype);
  }
  TM_LAUNCH_CHECK("k0_dequant launch");
  return TM_OK;
}

extern "C" int64_t tm_packed_w13_bytes(int hidden, int inter) { return 2LL * hidden * inter; }
extern "C" int64_t tm_packed_s13_floats(int hidden, int inter) { return 2LL * (inter / 128) * (hidden / 128); }
extern "C" int64_t tm_packed_w2_bytes(int hidden, int inter) { return (int64_t)hidden * inter; }
extern "C" int64_t tm_packed_s2_floats(int hidden, int inter) { return (int64_t)(hidden / 128) * (inter / 128); }

extern "C" int tm_pack_experts(const uint8_t *gate, const float *gate_s, const uint8_t *up,
                               const float *up_s, const uint8_t *down, const float *down_s,
                               int n_experts, int hidden, int inter, uint8_t *w13, float *s13,
                               uint8_t *w2, float *s2, void *stream) {
  TM_REQUIRE(gate && gate_s && up && up_s && down && down_s && w13 && s13 && w2 && s2, "null pointer");
  TM_REQUIRE(n_experts >= 1, "n_experts must be >= 1");
  TM_REQUIRE(hidden % 128 == 0 && inter % 128 == 0 && hidden > 0 && inter > 0,
             "hidden (%d) and inter (%d) must be positive multiples of 128", hidden, inter);
  TM_REQUIRE(aligned(gate, 16) && aligned(up, 16) && aligned(down, 16) && aligned(w13, 16) && aligned(w2, 16),
             "weight pointers must be 16-byte aligned");
  cudaStream_t s = as_stream(stream);
  const int threads = 256;
  const int64_t n = n_experts;
  k5_pack_w13<<<grid_for(n * inter * (hidden / 16) * 2, threads), threads, 0, s>>>(gate, up, n_experts,
                                                                                  hidden, inter, w13);
  TM_LAUNCH_CHECK("k5_pack_w13");
  k5_pack_s13<<<grid_for(n * tm_packed_s13_floats(hidden, inter), threads), threads, 0, s>>>(
      gate_s, up_s, n_experts, hidden, inter, s13);
  TM_LAUNCH_CHECK("k5_pack_s13");
  k5_pack_w2<<<grid_for(n * hidden * (inter / 16), threads), threads, 0, s>>>(down, n_experts, hidden,
                                                                              inter, w2);
  TM_LAUNCH_CHECK("k5_pack_w2");
  return cuda_check(cudaMemcpyAsync(s2, down_s, sizeof(float) * n * tm_packed_s2_floats(hidden, inter),
                                    cudaMemcpyDeviceToDevice, s),
                    "k5 s2 copy");
}

extern "C" int tm_pack_linear(const uint8_t *w, int out_features, int in_features, uint8_t *w_packed,
                              void *stream) {
  TM_REQUIRE(w && w_packed, "null pointer");
  TM_REQUIRE(out_features % 128 == 0 && in_features % 128 == 0 && out_features > 0 && in_features > 0,
             "out_features (%d) and in_features (%d) must be positive multiples of 128", out_features, in_features);
  TM_REQUIRE(aligned(w, 16) && aligned(w_packed, 16), "weight pointers must be 16-byte aligned");
  const int threads = 256;
  // a dense [N, K] matrix packs exactly like one expert's down projection ([H, I])
  k5_pack_w2<<<grid_for((int64_t)out_features * (in_features / 16), threads), threads, 0, as_stream(stream)>>>(
      w, 1, out_features, in_features, w_packed);
  TM_LAUNCH_CHECK("k5_pack_w2 (linear)");
  return TM_OK;
}

namespace {
struct Unpack {
  const uint8_t *w13; const float *s13; const uint8_t *w2; const float *s2;
  int H, I; void *g, *u, *d; cudaStream_t s;
  template <typename TO> int run() {
    const int threads = 256;
    if (g) k5_unpack_w13<TO><<<grid_for((int64_t)I * H / 16, threads), threads, 0, s>>>(w13, s13, H, I, 0, (TO *)g);
    if (u) k5_unpack_w13<TO><<<grid_for((int64_t)I * H / 16, threads), threads, 0, s>>>(w13, s13, H, I, 1, (TO *)u);
    if (d) k5_unpack_w2<TO><<<grid_for((int64_t)I * H / 16, threads), threads, 0, s>>>(w2, s2, H, I, (TO *)d);
    TM_LAUNCH_CHECK("k5_unpack");
    return TM_OK;
  }
};
}  // namespace

extern "C" int tm_unpack_expert(const uint8_t *w13, const float *s13, const uint8_t *w2,
                                const float *s2, int hidden, int inter, void *gate_out,
                                void *up_out, void *down_out, int out_dtype, void *stream) {
  TM_REQUIRE(w13 && s13 && w2 && s2, "null packed pointer");
  TM_REQUIRE(hidden % 128 == 0 && inter % 128 == 0 && hidden > 0 && inter > 0,
             "hidden and inter must be positive multiples of 128");
  TM_REQUIRE(aligned(w13, 16) && aligned(w2, 16), "packed weights must be 16-byte aligned");
  TM_REQUIRE((!gate_out || aligned(gate_out, 16)) && (!up_out || aligned(up_out, 16)) &&
                 (!down_out || aligned(down_out, 16)),
             "outputs must be 16-byte aligned");
  Unpack f{w13, s13, w2, s2, hidden, inter, gate_out, up_out, down_out, as_stream(stream)};
  return dispatch_act(out_dtype, f);
}

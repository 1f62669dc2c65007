// Attention-path glue of the TriFusion block: rotary q/k with the FP32
// attention operands written directly, and the pooled-grid interpolation.
//
//   rotary_qkv:  x [B, T, 3, H, D] (the qkv projection, BF16) ->
//                y [3, B, H, T, D] FP32 holding BF16 values: q and k rotated by
//                (a cos - b sin, a sin + b cos) on adjacent pairs with the
//                table angle of (t, pair), v copied
//                (kernels/primitives.py:116-150 `_rotary_qkv`; attention.py:14-16
//                widens its BF16 output to FP32 for the attention itself);
//   interpolate: y[b, t] = t < len ? a + (z - a) alpha : 0 with a, z the pooled
//                rows left[b, t], right[b, t] (kernels/native.py:103-138
//                `_interpolate`, `interpolate`; masking.py:71-80).
#include <cstdint>

#include "../../include/trifusion_b200.h"
#include "tf_common.cuh"
#include "tf_host.cuh"

namespace tf {
namespace {

constexpr int kThreads = 256;

int grid_for(int64_t items) {
  const int64_t blocks = (items + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

// One thread per (which, b, h, t, pair): two output elements.
__global__ void __launch_bounds__(kThreads) rotary_qkv_kernel(const bf16* __restrict__ x,
                                                              const float* __restrict__ cosv,
                                                              const float* __restrict__ sinv,
                                                              float* __restrict__ y, int B, int T, int H,
                                                              int D) {
  const int half = D / 2;
  const int64_t total = 3ll * B * H * T * half;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int pr = static_cast<int>(i % half);
    int64_t r = i / half;
    const int t = static_cast<int>(r % T);
    r /= T;
    const int h = static_cast<int>(r % H);
    r /= H;
    const int b = static_cast<int>(r % B);
    const int which = static_cast<int>(r / B);
    const int64_t src = (((static_cast<int64_t>(b) * T + t) * 3 + which) * H + h) * D + 2 * pr;
    const float2 v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(x + src));
    float u0 = v.x, u1 = v.y;
    if (which < 2) {
      const float cs = cosv[static_cast<int64_t>(t) * half + pr], sn = sinv[static_cast<int64_t>(t) * half + pr];
      // Separately rounded products and sums, as the reference kernel computes them.
      u0 = bf16_round(__fsub_rn(__fmul_rn(v.x, cs), __fmul_rn(v.y, sn)));
      u1 = bf16_round(__fadd_rn(__fmul_rn(v.x, sn), __fmul_rn(v.y, cs)));
    }
    *reinterpret_cast<float2*>(y + (i / half) * D + 2 * pr) = make_float2(u0, u1);
  }
}

// One thread per (b, t, 4 channels).
__global__ void __launch_bounds__(kThreads) interpolate_kernel(const bf16* __restrict__ low,
                                                               const int64_t* __restrict__ left,
                                                               const int64_t* __restrict__ right,
                                                               const float* __restrict__ alpha,
                                                               const int64_t* __restrict__ lengths,
                                                               bf16* __restrict__ y, int B, int T, int LT,
                                                               int D) {
  const int quads = D / 4;
  const int64_t total = static_cast<int64_t>(B) * T * quads;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int c = 4 * static_cast<int>(i % quads);
    const int64_t row = i / quads;  // b * T + t
    const int t = static_cast<int>(row % T);
    const int b = static_cast<int>(row / T);
    uint2 out = make_uint2(0, 0);
    if (t < lengths[b]) {
      const float al = alpha[row];
      int64_t lr = left[row], rr = right[row];
      lr = lr < 0 ? 0 : (lr >= LT ? LT - 1 : lr);  // grid indices lie in [0, LT) by construction;
      rr = rr < 0 ? 0 : (rr >= LT ? LT - 1 : rr);  // clamped so that no input can read outside it
      const uint2 ua = *reinterpret_cast<const uint2*>(low + (static_cast<int64_t>(b) * LT + lr) * D + c);
      const uint2 uz = *reinterpret_cast<const uint2*>(low + (static_cast<int64_t>(b) * LT + rr) * D + c);
      const float2 a0 = unpack_bf16x2(ua.x), a1 = unpack_bf16x2(ua.y);
      const float2 z0 = unpack_bf16x2(uz.x), z1 = unpack_bf16x2(uz.y);
      auto lerp = [al](float a, float z) { return __fadd_rn(a, __fmul_rn(__fsub_rn(z, a), al)); };
      out = make_uint2(pack_bf16x2(lerp(a0.x, z0.x), lerp(a0.y, z0.y)), pack_bf16x2(lerp(a1.x, z1.x), lerp(a1.y, z1.y)));
    }
    *reinterpret_cast<uint2*>(y + row * D + c) = out;
  }
}

// ---------------------------------------------------------------------------
// Attention over the pooled rows of one block (model.py:127-133 `GlobalAttention`
// after the qkv projection; kernels/primitives.py:116-150 rotary; attention.py:8-18
// FP32 masked attention): per batch entry b and head h,
//   q, k = rotary(qkv[b, :, 0|1, h]) rounded to BF16 (as rotary_qkv_kernel),
//   y[b, i, 64 h + d] = sum_{j < low_len[b]} softmax_j(q_i . k_j / 8) v[b, j, h, d],
// FP32 throughout, rounded once to BF16 in the [B, LT, H*64] row layout the out
// projection reads. One CTA per (64-row query tile, head, batch): warp w owns query
// rows 8w..8w+7 of the tile and treats them together (lane l scores key l against all
// 8); keys come in tiles of 32 with an online softmax; keys past the length are never
// loaded (their weight is exactly 0).
// ---------------------------------------------------------------------------
constexpr int kAttnD = 64;
constexpr int kAttnRows = 64;  // query rows per CTA
constexpr int kAttnKeys = 32;  // keys per tile

__global__ void __launch_bounds__(256) pooled_attention_kernel(const bf16* __restrict__ x,
                                                               const float* __restrict__ cosv,
                                                               const float* __restrict__ sinv,
                                                               const int64_t* __restrict__ lengths,
                                                               bf16* __restrict__ y, int LT, int H) {
  __shared__ __align__(16) float qs[kAttnRows][kAttnD];
  __shared__ float ks[kAttnKeys][kAttnD + 1];
  __shared__ float vs[kAttnKeys][kAttnD];
  const int tile = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int half = kAttnD / 2;
  int64_t len = lengths[b];
  if (len > LT) len = LT;
  if (len < 0) len = 0;
  const int64_t row_stride = 3ll * H * kAttnD;
  const bf16* xb = x + static_cast<int64_t>(b) * LT * row_stride;
  auto rotated = [&](int t, int which, int pr) -> float2 {
    const float2 v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(
        xb + t * row_stride + (static_cast<int64_t>(which) * H + h) * kAttnD + 2 * pr));
    const float cs = cosv[static_cast<int64_t>(t) * half + pr], sn = sinv[static_cast<int64_t>(t) * half + pr];
    return make_float2(bf16_round(__fsub_rn(__fmul_rn(v.x, cs), __fmul_rn(v.y, sn))),
                       bf16_round(__fadd_rn(__fmul_rn(v.x, sn), __fmul_rn(v.y, cs))));
  };
  for (int e = tid; e < kAttnRows * half; e += 256) {
    const int r = e / half, pr = e % half;
    const int t = tile * kAttnRows + r;
    const float2 q = t < LT ? rotated(t, 0, pr) : make_float2(0.f, 0.f);
    qs[r][2 * pr] = q.x;
    qs[r][2 * pr + 1] = q.y;
  }
  // Warp w owns rows 8w..8w+7 of the tile; a warp whose rows all lie past LT only
  // helps stage the key tiles.
  const int row0 = warp * 8;
  const bool active = tile * kAttnRows + row0 < LT;
  float m[8], l[8], o0[8], o1[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) { m[r] = -INFINITY; l[r] = 0.f; o0[r] = 0.f; o1[r] = 0.f; }
  for (int k0 = 0; k0 < len; k0 += kAttnKeys) {
    __syncthreads();  // previous tile consumed (and, the first time, the q tile written)
    for (int e = tid; e < kAttnKeys * half; e += 256) {
      const int j = e / half, pr = e % half;
      const int t = k0 + j;
      const float2 k = t < len ? rotated(t, 1, pr) : make_float2(0.f, 0.f);
      ks[j][2 * pr] = k.x;
      ks[j][2 * pr + 1] = k.y;
      float2 v = make_float2(0.f, 0.f);
      if (t < len)
        v = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(xb + t * row_stride + (2ll * H + h) * kAttnD + 2 * pr));
      vs[j][2 * pr] = v.x;
      vs[j][2 * pr + 1] = v.y;
    }
    __syncthreads();
    if (!active) continue;  // warp-uniform; the barriers above are still reached
    const bool valid = k0 + lane < len;
    // Scores of key `lane` against the warp's 8 rows: 8 independent FMA chains, one
    // read of the key's column per step (q rows are broadcast reads).
    float s[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) s[r] = 0.f;
#pragma unroll 4
    for (int d = 0; d < kAttnD; d += 4) {
      const float k0v = ks[lane][d], k1v = ks[lane][d + 1], k2v = ks[lane][d + 2], k3v = ks[lane][d + 3];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float4 q = *reinterpret_cast<const float4*>(&qs[row0 + r][d]);
        s[r] = fmaf(q.x, k0v, s[r]);
        s[r] = fmaf(q.y, k1v, s[r]);
        s[r] = fmaf(q.z, k2v, s[r]);
        s[r] = fmaf(q.w, k3v, s[r]);
      }
    }
    float mt[8], p[8], ps[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      s[r] = valid ? s[r] * 0.125f : -INFINITY;
      mt[r] = s[r];
    }
#pragma unroll
    for (int w = 16; w > 0; w >>= 1) {
#pragma unroll
      for (int r = 0; r < 8; ++r) mt[r] = fmaxf(mt[r], __shfl_xor_sync(0xffffffffu, mt[r], w));
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const float mn = fmaxf(m[r], mt[r]);  // finite: this tile holds at least one valid key
      const float scale = m[r] == -INFINITY ? 0.f : expf(m[r] - mn);
      p[r] = valid ? expf(s[r] - mn) : 0.f;
      ps[r] = p[r];
      m[r] = mn;
      l[r] *= scale;
      o0[r] *= scale;
      o1[r] *= scale;
    }
#pragma unroll
    for (int w = 16; w > 0; w >>= 1) {
#pragma unroll
      for (int r = 0; r < 8; ++r) ps[r] += __shfl_xor_sync(0xffffffffu, ps[r], w);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) l[r] += ps[r];
    // Weighted values: each v row is read once for all 8 rows.
#pragma unroll 4
    for (int j = 0; j < kAttnKeys; ++j) {
      const float v0 = vs[j][lane], v1 = vs[j][lane + 32];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float pj = __shfl_sync(0xffffffffu, p[r], j);
        o0[r] = fmaf(pj, v0, o0[r]);
        o1[r] = fmaf(pj, v1, o1[r]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int t = tile * kAttnRows + warp * 8 + r;
    if (t >= LT) break;
    // No valid key (length 0): NaN, as the reference's softmax over an all-masked row.
    const float inv = l[r] > 0.f ? 1.f / l[r] : __int_as_float(0x7fc00000);
    bf16* yr = y + (static_cast<int64_t>(b) * LT + t) * H * kAttnD + h * kAttnD;
    yr[lane] = __float2bfloat16_rn(o0[r] * inv);
    yr[lane + 32] = __float2bfloat16_rn(o1[r] * inv);
  }
}

}  // namespace
}  // namespace tf

extern "C" {

int tf_pooled_attention_fwd(const void* x, const float* cosv, const float* sinv, const int64_t* lengths, void* y,
                            int batch, int low_time, int heads, int head_dim, void* stream) {
  if (batch < 0 || low_time < 0 || heads < 0 || head_dim != tf::kAttnD) return TF_ERR_ARG;
  if (batch == 0 || low_time == 0 || heads == 0) return TF_OK;
  if (!x || !cosv || !sinv || !lengths || !y) return TF_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 4) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const dim3 grid((low_time + tf::kAttnRows - 1) / tf::kAttnRows, heads, batch);
  tf::pooled_attention_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const tf::bf16*>(x), cosv, sinv, lengths, static_cast<tf::bf16*>(y), low_time, heads);
  return tf::launch_status();
}

int tf_rotary_qkv_fwd(const void* x, const float* cosv, const float* sinv, float* y, int batch,
                      int time, int heads, int head_dim, void* stream) {
  if (batch < 0 || time < 0 || heads < 0 || head_dim <= 0 || head_dim % 2) return TF_ERR_ARG;
  if (batch == 0 || time == 0 || heads == 0) return TF_OK;
  if (!x || !cosv || !sinv || !y) return TF_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 4 || reinterpret_cast<uintptr_t>(y) % 8) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const int64_t items = 3ll * batch * heads * time * (head_dim / 2);
  tf::rotary_qkv_kernel<<<tf::grid_for(items), tf::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const tf::bf16*>(x), cosv, sinv, y, batch, time, heads, head_dim);
  return tf::launch_status();
}

int tf_interpolate_fwd(const void* low, const int64_t* left, const int64_t* right, const float* alpha,
                       const int64_t* lengths, void* y, int batch, int time, int low_time, int width,
                       void* stream) {
  if (batch < 0 || time < 0 || low_time < 0 || width < 0) return TF_ERR_ARG;
  if (width % 4) return TF_ERR_LAYOUT;
  if (batch == 0 || time == 0 || width == 0) return TF_OK;
  if (!low || !left || !right || !alpha || !lengths || !y || low_time == 0) return TF_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(low) % 8 || reinterpret_cast<uintptr_t>(y) % 8) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const int64_t items = static_cast<int64_t>(batch) * time * (width / 4);
  tf::interpolate_kernel<<<tf::grid_for(items), tf::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const tf::bf16*>(low), left, right, alpha, lengths, static_cast<tf::bf16*>(y), batch, time,
      low_time, width);
  return tf::launch_status();
}

}  // extern "C"

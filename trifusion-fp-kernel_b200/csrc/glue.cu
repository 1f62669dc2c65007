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

}  // namespace
}  // namespace tf

extern "C" {

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

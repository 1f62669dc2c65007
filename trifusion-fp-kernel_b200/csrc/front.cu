// Spectrogram front-end passes around the cuDNN convolutions, on channels-last
// (NHWC) activations: a [B, C, T, F] tensor stored as [B, T, F, C], so every
// (b, t, f) position is one contiguous row of C channels.
//
//   front norm:     y = t < len ? RMSNorm_C(x) * w : 0, then optionally SiLU
//                   (kernels/primitives.py:153-187 `_front_norm`, kernels/buffers.py:58-79);
//   residual tail:  y = t < len ? silu(h + skip) : 0   (front.py:43);
//   bands:          y[b, t, band, c] = mean of x[b, t, f, c] over the band's
//                   frequencies [floor(band F / 8), ceil((band + 1) F / 8))
//                   (kernels/native.py:141-163 `_bands`; front.py:80-87).
// Rounding follows the reference: BF16 results are rounded once where the
// reference stores a BF16 tensor (the normalised value before SiLU, the
// residual sum before SiLU).
#include <cstdint>

#include "../../include/trifusion_b200.h"
#include "tf_common.cuh"
#include "tf_host.cuh"

namespace tf {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float to_f(float v) { return v; }
__device__ __forceinline__ float to_f(bf16 v) { return __bfloat162float(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v);
template <>
__device__ __forceinline__ float from_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ bf16 from_f<bf16>(float v) { return __float2bfloat16_rn(v); }
// The value a tensor of type T would hold.
template <typename T>
__device__ __forceinline__ float round_to(float v) { return to_f(from_f<T>(v)); }

__device__ __forceinline__ float sigmoid_ieee(float x) { return 1.f / (1.f + expf(-x)); }

__device__ __forceinline__ int valid_len(const int64_t* lengths, int b, int T) {
  const int64_t len = lengths[b];
  return static_cast<int>(len < 0 ? 0 : (len > T ? T : len));
}

int grid_for(int64_t items, int per_block) {
  const int64_t blocks = (items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

// One warp per (b, t, f) row of C channels; C <= 32 * kMaxPerLane.
template <typename T, int kMaxPerLane>
__global__ void __launch_bounds__(kThreads) front_norm_kernel(const T* __restrict__ x,
                                                              const float* __restrict__ w,
                                                              const int64_t* __restrict__ lengths,
                                                              T* __restrict__ y, int B, int Tn, int F,
                                                              int C, float eps, int silu) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(B) * Tn * F;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  for (int64_t row = blockIdx.x * static_cast<int64_t>(kThreads / 32) + (threadIdx.x >> 5); row < rows;
       row += warps) {
    const int t = static_cast<int>((row / F) % Tn);
    const int b = static_cast<int>(row / (static_cast<int64_t>(F) * Tn));
    const bool live = t < valid_len(lengths, b, Tn);
    const T* xr = x + row * C;
    float v[kMaxPerLane];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int ch = lane + 32 * i;
      v[i] = (live && ch < C) ? to_f(xr[ch]) : 0.f;
      ss = fmaf(v[i], v[i], ss);
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(C) + eps);
    T* yr = y + row * C;
#pragma unroll
    for (int i = 0; i < kMaxPerLane; ++i) {
      const int ch = lane + 32 * i;
      if (ch < C) {
        float o = round_to<T>(v[i] * r * w[ch]);
        if (silu) o = o * sigmoid_ieee(o);
        yr[ch] = from_f<T>(o);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) residual_silu_kernel(const T* __restrict__ h,
                                                                 const T* __restrict__ skip,
                                                                 const int64_t* __restrict__ lengths,
                                                                 T* __restrict__ y, int B, int Tn, int F,
                                                                 int C) {
  const int64_t total = static_cast<int64_t>(B) * Tn * F * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t row = i / C;
    const int t = static_cast<int>((row / F) % Tn);
    const int b = static_cast<int>(row / (static_cast<int64_t>(F) * Tn));
    float o = 0.f;
    if (t < valid_len(lengths, b, Tn)) {
      const float s = round_to<T>(to_f(h[i]) + to_f(skip[i]));
      o = s * sigmoid_ieee(s);
    }
    y[i] = from_f<T>(o);
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) bands_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                         int B, int Tn, int F, int C) {
  const int64_t total = static_cast<int64_t>(B) * Tn * 8 * C;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int c = static_cast<int>(i % C);
    const int band = static_cast<int>((i / C) % 8);
    const int64_t bt = i / (static_cast<int64_t>(C) * 8);
    const int start = band * F / 8, end = ((band + 1) * F + 7) / 8;
    const T* xr = x + bt * F * C + c;
    float acc = 0.f;
    for (int f = start; f < end; ++f) acc += to_f(xr[static_cast<int64_t>(f) * C]);
    y[i] = from_f<T>(acc / static_cast<float>(end - start));
  }
}

template <typename T>
int launch_front_norm(const void* x, const float* w, const int64_t* lengths, void* y, int B, int Tn,
                      int F, int C, float eps, int silu, cudaStream_t s) {
  const int64_t rows = static_cast<int64_t>(B) * Tn * F;
  const int grid = grid_for(rows, kThreads / 32);
  auto X = static_cast<const T*>(x);
  auto Y = static_cast<T*>(y);
  if (C <= 32)
    front_norm_kernel<T, 1><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, C, eps, silu);
  else if (C <= 64)
    front_norm_kernel<T, 2><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, C, eps, silu);
  else if (C <= 128)
    front_norm_kernel<T, 4><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, C, eps, silu);
  else
    front_norm_kernel<T, 8><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, C, eps, silu);
  return launch_status();
}

}  // namespace
}  // namespace tf

extern "C" {

int tf_front_norm_fwd(const void* x, int dtype, const float* w, const int64_t* lengths, void* y,
                      int batch, int time, int freq, int channels, float eps, int silu, void* stream) {
  if (batch < 0 || time < 0 || freq < 0 || channels <= 0) return TF_ERR_ARG;
  if (dtype != TF_F32 && dtype != TF_BF16) return TF_ERR_ARG;
  if (channels > 256) return TF_ERR_SIZE;
  if (batch == 0 || time == 0 || freq == 0) return TF_OK;
  if (!x || !w || !lengths || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F32)
    return tf::launch_front_norm<float>(x, w, lengths, y, batch, time, freq, channels, eps, silu, s);
  return tf::launch_front_norm<tf::bf16>(x, w, lengths, y, batch, time, freq, channels, eps, silu, s);
}

int tf_front_residual_fwd(const void* h, const void* skip, int dtype, const int64_t* lengths, void* y,
                          int batch, int time, int freq, int channels, void* stream) {
  if (batch < 0 || time < 0 || freq < 0 || channels < 0) return TF_ERR_ARG;
  if (dtype != TF_F32 && dtype != TF_BF16) return TF_ERR_ARG;
  if (batch == 0 || time == 0 || freq == 0 || channels == 0) return TF_OK;
  if (!h || !skip || !lengths || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = tf::grid_for(static_cast<int64_t>(batch) * time * freq * channels, tf::kThreads);
  if (dtype == TF_F32)
    tf::residual_silu_kernel<float><<<grid, tf::kThreads, 0, s>>>(
        static_cast<const float*>(h), static_cast<const float*>(skip), lengths, static_cast<float*>(y),
        batch, time, freq, channels);
  else
    tf::residual_silu_kernel<tf::bf16><<<grid, tf::kThreads, 0, s>>>(
        static_cast<const tf::bf16*>(h), static_cast<const tf::bf16*>(skip), lengths,
        static_cast<tf::bf16*>(y), batch, time, freq, channels);
  return tf::launch_status();
}

int tf_bands_fwd(const void* x, int dtype, void* y, int batch, int time, int freq, int channels,
                 void* stream) {
  if (batch < 0 || time < 0 || freq <= 0 || channels < 0) return TF_ERR_ARG;
  if (dtype != TF_F32 && dtype != TF_BF16) return TF_ERR_ARG;
  if (batch == 0 || time == 0 || channels == 0) return TF_OK;
  if (!x || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = tf::grid_for(static_cast<int64_t>(batch) * time * 8 * channels, tf::kThreads);
  if (dtype == TF_F32)
    tf::bands_kernel<float><<<grid, tf::kThreads, 0, s>>>(static_cast<const float*>(x),
                                                          static_cast<float*>(y), batch, time, freq,
                                                          channels);
  else
    tf::bands_kernel<tf::bf16><<<grid, tf::kThreads, 0, s>>>(static_cast<const tf::bf16*>(x),
                                                             static_cast<tf::bf16*>(y), batch, time,
                                                             freq, channels);
  return tf::launch_status();
}

}  // extern "C"

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

// Streaming kernels: enough resident threads for many 16-byte requests in flight.
int grid_vec(int64_t threads) {
  const int64_t blocks = (threads + kThreads - 1) / kThreads;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 16;
  return static_cast<int>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

int grid_for(int64_t items, int per_block) {
  const int64_t blocks = (items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

// A group of G = C / 8 threads per (b, t, f) row; each thread moves one 16-byte
// vector of 8 BF16 channels and the group reduces with shuffles. Used for BF16
// rows with C in {8, 16, 32, 64, 128, 256}.
template <int G>
__global__ void __launch_bounds__(kThreads) front_norm_vec_kernel(const bf16* __restrict__ x,
                                                                  const float* __restrict__ w,
                                                                  const int64_t* __restrict__ lengths,
                                                                  bf16* __restrict__ y, int B, int Tn, int F,
                                                                  float eps, int silu) {
  constexpr int C = 8 * G;
  const int64_t rows = static_cast<int64_t>(B) * Tn * F;
  const int sub = threadIdx.x % G;
  const float4 w0 = *reinterpret_cast<const float4*>(w + 8 * sub);
  const float4 w1 = *reinterpret_cast<const float4*>(w + 8 * sub + 4);
  const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
  const int64_t stride = static_cast<int64_t>(gridDim.x) * (kThreads / G);
  // The loop bound is uniform across the block, so whole warps take part in the
  // group shuffles; rows past the end only skip their loads and stores.
  for (int64_t first = blockIdx.x * static_cast<int64_t>(kThreads / G); first < rows; first += stride) {
    const int64_t row = first + threadIdx.x / G;
    const bool in = row < rows;
    bool live = false;
    if (in) {
      const int t = static_cast<int>((row / F) % Tn);
      const int b = static_cast<int>(row / (static_cast<int64_t>(F) * Tn));
      live = t < valid_len(lengths, b, Tn);
    }
    float v[8];
    if (live) {
      const uint4 u = *reinterpret_cast<const uint4*>(x + row * C + 8 * sub);
      const uint32_t ww[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f2 = unpack_bf16x2(ww[i]);
        v[2 * i] = f2.x;
        v[2 * i + 1] = f2.y;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
    for (int o = 1; o < G; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float r = rsqrtf(ss / static_cast<float>(C) + eps);
    uint32_t out[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = round_to<bf16>(v[2 * i] * r * wv[2 * i]);
      float c = round_to<bf16>(v[2 * i + 1] * r * wv[2 * i + 1]);
      if (silu) {
        a = a * sigmoid_ieee(a);
        c = c * sigmoid_ieee(c);
      }
      out[i] = pack_bf16x2(a, c);
    }
    if (in) *reinterpret_cast<uint4*>(y + row * C + 8 * sub) = make_uint4(out[0], out[1], out[2], out[3]);
  }
}

// Stem of the first CNN stage (front.py:8-43 with C_in = 1, C_out = 32, time stride
// 1; front.py:21,33,43): the 3x3 convolution (stride (1, 2), zero padding 1) and the 1x1 skip
// (stride (1, 2)) of the [B, T, F] spectrogram, computed as the BF16 autocast
// convolutions do (inputs and weights rounded to BF16, FP32 accumulation, BF16
// result), then the conv branch's masked channel RMSNorm and SiLU in the rounding
// and summation order of front_norm_vec_kernel<4>. One thread per output position,
// its 32 channels in registers; both outputs channels-last [B, T, F2, 32] BF16.
constexpr int kStemC = 32;
__global__ void __launch_bounds__(kThreads, 2) front_stem_kernel(const float* __restrict__ x,
                                                              const float* __restrict__ w1,
                                                              const float* __restrict__ ws,
                                                              const float* __restrict__ nw,
                                                              const int64_t* __restrict__ lengths,
                                                              bf16* __restrict__ h, bf16* __restrict__ sk, int B,
                                                              int Tn, int F, int F2, float eps) {
  // 3x3 weights padded to 12 per channel: three 16-byte shared loads per channel.
  __shared__ __align__(16) float s_w1[kStemC * 12];
  __shared__ __align__(16) float s_ws[kStemC];
  __shared__ __align__(16) float s_nw[kStemC];
  for (int i = threadIdx.x; i < kStemC * 12; i += kThreads) {
    const int c = i / 12, k = i - 12 * (i / 12);
    s_w1[i] = k < 9 ? round_to<bf16>(w1[c * 9 + k]) : 0.f;
  }
  if (threadIdx.x < kStemC) {
    s_ws[threadIdx.x] = round_to<bf16>(ws[threadIdx.x]);
    s_nw[threadIdx.x] = nw[threadIdx.x];
  }
  __syncthreads();
  const int64_t positions = static_cast<int64_t>(B) * Tn * F2;
  for (int64_t pos = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; pos < positions;
       pos += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int f2 = static_cast<int>(pos % F2);
    const int64_t bt = pos / F2;
    const int t = static_cast<int>(bt % Tn);
    const int b = static_cast<int>(bt / Tn);
    float xin[9];
#pragma unroll
    for (int dt = 0; dt < 3; ++dt) {
      const int tt = t + dt - 1;
#pragma unroll
      for (int df = 0; df < 3; ++df) {
        const int ff = 2 * f2 + df - 1;
        xin[3 * dt + df] = (tt >= 0 && tt < Tn && ff >= 0 && ff < F)
                               ? round_to<bf16>(x[(static_cast<int64_t>(b) * Tn + tt) * F + ff])
                               : 0.f;
      }
    }
    // Skip: one exact product per channel, rounded to BF16.
    uint32_t so[kStemC / 2];
#pragma unroll
    for (int c = 0; c < kStemC; c += 4) {
      const float4 w4 = *reinterpret_cast<const float4*>(&s_ws[c]);
      so[c / 2] = pack_bf16x2(xin[4] * w4.x, xin[4] * w4.y);
      so[c / 2 + 1] = pack_bf16x2(xin[4] * w4.z, xin[4] * w4.w);
    }
    bf16* srow = sk + pos * kStemC;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4*>(srow + 8 * q) = make_uint4(so[4 * q], so[4 * q + 1], so[4 * q + 2], so[4 * q + 3]);
    // Conv branch, then the norm (zero rows past the length) and SiLU.
    const bool live = t < valid_len(lengths, b, Tn);
    float v[kStemC];
#pragma unroll
    for (int c = 0; c < kStemC; ++c) {
      const float4 wa = *reinterpret_cast<const float4*>(&s_w1[c * 12]);
      const float4 wb = *reinterpret_cast<const float4*>(&s_w1[c * 12 + 4]);
      const float4 wc = *reinterpret_cast<const float4*>(&s_w1[c * 12 + 8]);
      const float wk[9] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w, wc.x};
      float acc = 0.f;
#pragma unroll
      for (int k = 0; k < 9; ++k) acc = fmaf(xin[k], wk[k], acc);
      v[c] = live ? round_to<bf16>(acc) : 0.f;
    }
    float g[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      g[q] = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) g[q] = fmaf(v[8 * q + i], v[8 * q + i], g[q]);
    }
    const float ss = (g[0] + g[1]) + (g[2] + g[3]);
    const float r = rsqrtf(ss / static_cast<float>(kStemC) + eps);
    uint32_t ho[kStemC / 2];
#pragma unroll
    for (int c = 0; c < kStemC; c += 4) {
      const float4 n4 = *reinterpret_cast<const float4*>(&s_nw[c]);
      const float nw4[4] = {n4.x, n4.y, n4.z, n4.w};
#pragma unroll
      for (int e = 0; e < 4; e += 2) {
        float a = round_to<bf16>(v[c + e] * r * nw4[e]);
        float d = round_to<bf16>(v[c + e + 1] * r * nw4[e + 1]);
        a = a * sigmoid_ieee(a);
        d = d * sigmoid_ieee(d);
        ho[(c + e) / 2] = pack_bf16x2(a, d);
      }
    }
    bf16* hrow = h + pos * kStemC;
#pragma unroll
    for (int q = 0; q < 4; ++q)
      *reinterpret_cast<uint4*>(hrow + 8 * q) = make_uint4(ho[4 * q], ho[4 * q + 1], ho[4 * q + 2], ho[4 * q + 3]);
  }
}

// General form: one warp per row; C <= 32 * kMaxPerLane.
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

// BF16, C % 8 == 0: each thread handles one 16-byte vector of a row.
__global__ void __launch_bounds__(kThreads) residual_silu_vec_kernel(const bf16* __restrict__ h,
                                                                     const bf16* __restrict__ skip,
                                                                     const int64_t* __restrict__ lengths,
                                                                     bf16* __restrict__ y, int B, int Tn,
                                                                     int F, int C) {
  const int64_t vecs = static_cast<int64_t>(B) * Tn * F * (C / 8);
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < vecs;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t row = i / (C / 8);
    const int t = static_cast<int>((row / F) % Tn);
    const int b = static_cast<int>(row / (static_cast<int64_t>(F) * Tn));
    uint4 out = make_uint4(0, 0, 0, 0);
    if (t < valid_len(lengths, b, Tn)) {
      const uint4 a = reinterpret_cast<const uint4*>(h)[i];
      const uint4 c = reinterpret_cast<const uint4*>(skip)[i];
      const uint32_t aa[4] = {a.x, a.y, a.z, a.w}, cc[4] = {c.x, c.y, c.z, c.w};
      uint32_t o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 p = unpack_bf16x2(aa[k]), q = unpack_bf16x2(cc[k]);
        const float s0 = round_to<bf16>(p.x + q.x), s1 = round_to<bf16>(p.y + q.y);
        o[k] = pack_bf16x2(s0 * sigmoid_ieee(s0), s1 * sigmoid_ieee(s1));
      }
      out = make_uint4(o[0], o[1], o[2], o[3]);
    }
    reinterpret_cast<uint4*>(y)[i] = out;
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
  auto X = static_cast<const T*>(x);
  auto Y = static_cast<T*>(y);
  if constexpr (sizeof(T) == 2) {
    const bool vec = (C == 8 || C == 16 || C == 32 || C == 64 || C == 128 || C == 256) &&
                     reinterpret_cast<uintptr_t>(x) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(w) % 16 == 0;
    if (vec) {
      const int g = C / 8;
      const int grid = grid_vec(rows * g);
      switch (g) {
        case 1: front_norm_vec_kernel<1><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, eps, silu); break;
        case 2: front_norm_vec_kernel<2><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, eps, silu); break;
        case 4: front_norm_vec_kernel<4><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, eps, silu); break;
        case 8: front_norm_vec_kernel<8><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, eps, silu); break;
        case 16: front_norm_vec_kernel<16><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, eps, silu); break;
        default: front_norm_vec_kernel<32><<<grid, kThreads, 0, s>>>(X, w, lengths, Y, B, Tn, F, eps, silu); break;
      }
      return launch_status();
    }
  }
  const int grid = grid_for(rows, kThreads / 32);
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

int tf_front_stem_fwd(const float* x, const float* w1, const float* ws, const float* norm_w,
                      const int64_t* lengths, void* h, void* skip, int batch, int time, int freq, float eps,
                      void* stream) {
  if (batch < 0 || time < 0 || freq < 1) return TF_ERR_ARG;
  if (batch == 0 || time == 0) return TF_OK;
  if (!x || !w1 || !ws || !norm_w || !lengths || !h || !skip) return TF_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(h) % 16 || reinterpret_cast<uintptr_t>(skip) % 16) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const int f2 = (freq - 1) / 2 + 1;
  const int64_t positions = static_cast<int64_t>(batch) * time * f2;
  tf::front_stem_kernel<<<tf::grid_for(positions, tf::kThreads), tf::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      x, w1, ws, norm_w, lengths, static_cast<tf::bf16*>(h), static_cast<tf::bf16*>(skip), batch, time, freq, f2,
      eps);
  return tf::launch_status();
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
  if (dtype == TF_BF16 && channels % 8 == 0 && reinterpret_cast<uintptr_t>(h) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(skip) % 16 == 0 && reinterpret_cast<uintptr_t>(y) % 16 == 0) {
    const int64_t vecs = static_cast<int64_t>(batch) * time * freq * (channels / 8);
    tf::residual_silu_vec_kernel<<<tf::grid_vec(vecs), tf::kThreads, 0, s>>>(
        static_cast<const tf::bf16*>(h), static_cast<const tf::bf16*>(skip), lengths, static_cast<tf::bf16*>(y),
        batch, time, freq, channels);
    return tf::launch_status();
  }
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

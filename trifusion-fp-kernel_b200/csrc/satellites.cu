// Satellite operators around the recurrence: row norms, controls, length
// masking and reversal, SwiGLU, branch gate, pooling and decoder reads.
//
// All are HBM-bound element or row passes. Design rules used throughout:
//   * rows are contiguous; each warp (or thread) moves 16-byte vectors when the
//     row size and the base pointers allow it, else 8-, 4- or 2-byte ones;
//   * grids are sized to a few waves of the SM count and loop (grid-stride);
//   * arithmetic is FP32, results are rounded once to the output type;
//   * index and copy operators move raw bits (bit-exact by construction).
// The reference formula each kernel follows is cited at the kernel.
#include <cstdint>
#include <type_traits>
#include <cstdio>

#include "../../include/trifusion_b200.h"
#include "tf_common.cuh"
#include "tf_host.cuh"

namespace tf {
namespace {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ float load_f(const T* p);
template <>
__device__ __forceinline__ float load_f<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float load_f<bf16>(const bf16* p) { return __bfloat162float(*p); }

template <typename T>
__device__ __forceinline__ void store_f(T* p, float v);
template <>
__device__ __forceinline__ void store_f<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void store_f<bf16>(bf16* p, float v) { *p = __float2bfloat16_rn(v); }

// 4 consecutive elements as FP32 (8- or 16-byte load; caller guarantees alignment).
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const bf16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y);
  return make_float4(a.x, a.y, b.x, b.y);
}
__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(bf16* p, float4 v) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16x2(v.x, v.y), pack_bf16x2(v.z, v.w));
}

// IEEE sigmoid in FP32: 1 / (1 + e^-x), with expf and a correctly rounded divide.
__device__ __forceinline__ float sigmoid_ieee(float x) { return 1.f / (1.f + expf(-x)); }

int grid_for(int64_t work_items, int per_block) {
  const int64_t blocks = (work_items + per_block - 1) / per_block;
  const int64_t cap = static_cast<int64_t>(sm_count()) * 8;
  return static_cast<int>(blocks < 1 ? 1 : (blocks < cap ? blocks : cap));
}

bool aligned(const void* p, int bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

// ---------------------------------------------------------------------------
// Row RMSNorm family (kernels/native.py:8-39 `_norm`; kernels/primitives.py:8-22
// `_rms_fwd`). One warp per row:
//   kMode 0 (rms):           y = x * rsqrt(mean(x^2) + eps) * w      (y type = x type)
//   kMode 1 (evidence_norm): x' = x + a * 2 sigmoid(b) on rows whose mask is set,
//                            0 elsewhere; y = rms(x') * w            (FP32 out)
//   kMode 2 (mean_norm):     x' = (x + a) / 2; y = rms(x') * w       (FP32 out)
//   kMode 3 (rms + SiLU):    a = round(rms(x) * w); y = a / (1 + e^-a)  (PyTorch's silu on the
//                            norm's output tensor, model.py:120 `silu(self.norm(h))`)
//   kMode 4 (add + rms):     x' = x + a (FP32, a promoted exactly), written to xo; y = rms(x') * w
//                            (model.py:197-198 `r = x + merge(...)`, `ff_norm(r)`)
// The row is read twice (sum of squares, then scale); the second read hits L1.
// Output rows start every `yp` elements (0: every `width`), so a norm can write its
// slice of a concatenated row in place; `y2` (optional, BF16, rows every `y2p`)
// receives the same values rounded once, the copy autocast would make for a projection.
// The second and third inputs (a, b) may have their own row pitch `ap` (0: `width`),
// e.g. the two halves of one stacked projection row.
// ---------------------------------------------------------------------------
template <int kMode, typename TX, typename TA, typename TY, bool kVec4>
__global__ void __launch_bounds__(kThreads) row_norm_kernel(const TX* __restrict__ x,
                                                            const TA* __restrict__ a,
                                                            const TA* __restrict__ b,
                                                            const float* __restrict__ w,
                                                            const uint8_t* __restrict__ mask,
                                                            TY* __restrict__ y, int64_t rows,
                                                            int width, float eps, float* __restrict__ xo = nullptr,
                                                            int64_t yp = 0, bf16* __restrict__ y2 = nullptr,
                                                            int64_t y2p = 0, int64_t ap = 0) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  auto value = [&](int64_t off, int64_t aoff) -> float {
    float v = load_f(x + off);
    if (kMode == 1) v = v + load_f(a + aoff) * (2.f * sigmoid_ieee(load_f(b + aoff)));
    if (kMode == 2) v = (v + load_f(a + aoff)) * 0.5f;
    if (kMode == 4) v = v + load_f(a + aoff);
    return v;
  };
  auto value4 = [&](int64_t off, int64_t aoff) -> float4 {
    float4 v = load4(x + off);
    if (kMode == 1) {
      const float4 av = load4(a + aoff), bv = load4(b + aoff);
      v.x += av.x * (2.f * sigmoid_ieee(bv.x));
      v.y += av.y * (2.f * sigmoid_ieee(bv.y));
      v.z += av.z * (2.f * sigmoid_ieee(bv.z));
      v.w += av.w * (2.f * sigmoid_ieee(bv.w));
    }
    if (kMode == 2) {
      const float4 av = load4(a + aoff);
      v = make_float4((v.x + av.x) * 0.5f, (v.y + av.y) * 0.5f, (v.z + av.z) * 0.5f,
                      (v.w + av.w) * 0.5f);
    }
    if (kMode == 4) {
      const float4 av = load4(a + aoff);
      v = make_float4(v.x + av.x, v.y + av.y, v.z + av.z, v.w + av.w);
    }
    return v;
  };
  for (int64_t row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < rows; row += warps) {
    const int64_t base = row * width;
    const int64_t ybase = row * (yp ? yp : width);
    const int64_t abase = row * (ap ? ap : width);
    const bool live = kMode != 1 || mask[row] != 0;
    float ss = 0.f;
    if (live) {
      if (kVec4) {
        for (int c = lane * 4; c < width; c += 128) {
          const float4 v = value4(base + c, abase + c);
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
      } else {
        for (int c = lane; c < width; c += 32) {
          const float v = value(base + c, abase + c);
          ss += v * v;
        }
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / static_cast<float>(width) + eps);
    auto silu_of_rounded = [](float t) -> float {
      float a = t;
      if constexpr (!std::is_same<TY, float>::value) a = bf16_round(t);
      return a / (1.f + expf(-a));
    };
    if (kVec4) {
      for (int c = lane * 4; c < width; c += 128) {
        float4 v = live ? value4(base + c, abase + c) : make_float4(0.f, 0.f, 0.f, 0.f);
        if (kMode == 4) store4(xo + base + c, v);
        const float4 wv = load4(w + c);
        v = make_float4(v.x * r * wv.x, v.y * r * wv.y, v.z * r * wv.z, v.w * r * wv.w);
        if (kMode == 3)
          v = make_float4(silu_of_rounded(v.x), silu_of_rounded(v.y), silu_of_rounded(v.z), silu_of_rounded(v.w));
        store4(y + ybase + c, v);
        if (y2) store4(y2 + row * y2p + c, v);
      }
    } else {
      for (int c = lane; c < width; c += 32) {
        const float v = live ? value(base + c, abase + c) : 0.f;
        if (kMode == 4) xo[base + c] = v;
        const float t = v * r * w[c];
        store_f(y + ybase + c, kMode == 3 ? silu_of_rounded(t) : t);
        if (y2) store_f(y2 + row * y2p + c, t);
      }
    }
  }
}

template <int kMode, typename TX, typename TA, typename TY>
int launch_row_norm(const void* x, const void* a, const void* b, const float* w,
                    const uint8_t* mask, void* y, int64_t rows, int width, float eps,
                    cudaStream_t s, float* xo = nullptr, int64_t yp = 0, bf16* y2 = nullptr,
                    int64_t y2p = 0, int64_t ap = 0) {
  const bool v4 = width % 4 == 0 && aligned(x, 4 * sizeof(TX)) && aligned(y, 4 * sizeof(TY)) &&
                  aligned(w, 16) && (kMode == 0 || aligned(a, 4 * sizeof(TA))) &&
                  (kMode != 1 || aligned(b, 4 * sizeof(TA))) && yp % 4 == 0 && ap % 4 == 0 &&
                  (!y2 || (aligned(y2, 8) && y2p % 4 == 0));
  const int grid = grid_for(rows, kThreads / 32);
  auto X = static_cast<const TX*>(x);
  auto A = static_cast<const TA*>(a);
  auto B = static_cast<const TA*>(b);
  auto Y = static_cast<TY*>(y);
  if (v4)
    row_norm_kernel<kMode, TX, TA, TY, true><<<grid, kThreads, 0, s>>>(X, A, B, w, mask, Y, rows, width, eps, xo,
                                                                      yp, y2, y2p, ap);
  else
    row_norm_kernel<kMode, TX, TA, TY, false><<<grid, kThreads, 0, s>>>(X, A, B, w, mask, Y, rows, width, eps, xo,
                                                                       yp, y2, y2p, ap);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Mamba controls (kernels/primitives.py:190-216 `_controls`, called from
// kernels/buffers.py:82-101; the PyTorch form is mamba.py:58-63):
//   A   = min(-(max(a, 0) + 1 / (1 - min(a, 0))), -floor)
//   dt  = softplus(ddt + bias[h])   (identity above 20)
//   out: adt = A * dt and dt, transposed from [B, T, H] to [B, H, T].
// One thread per output element, t fastest, so the stores are coalesced; the
// strided reads of the projection view are a few bytes per token.
// ---------------------------------------------------------------------------
template <typename TI>
__global__ void __launch_bounds__(kThreads) controls_kernel(const TI* __restrict__ a,
                                                            const TI* __restrict__ ddt,
                                                            int64_t sab, int64_t sat,
                                                            int64_t sdb, int64_t sdtt,
                                                            const float* __restrict__ bias,
                                                            float floor_, float* __restrict__ adt,
                                                            float* __restrict__ dt, int B, int T,
                                                            int H) {
  const int64_t total = static_cast<int64_t>(B) * H * T;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int t = static_cast<int>(i % T);
    const int64_t bh = i / T;
    const int h = static_cast<int>(bh % H);
    const int b = static_cast<int>(bh / H);
    const float av = load_f(a + b * sab + t * sat + h);
    const float dv = load_f(ddt + b * sdb + t * sdtt + h);
    const float control = fminf(-(fmaxf(av, 0.f) + 1.f / (1.f - fminf(av, 0.f))), -floor_);
    const float v = dv + bias[h];
    const float step = v > 20.f ? v : log1pf(expf(v));
    dt[i] = step;
    adt[i] = control * step;
  }
}

// ---------------------------------------------------------------------------
// Raw-bit row operators. `V` is the vector type (uint4/uint2/uint32_t/uint16_t)
// that divides the row size and both base pointers.
// ---------------------------------------------------------------------------

// Length mask (kernels/primitives.py:65-70 `_mask`, kernels/buffers.py:6-10;
// masking.py:10-11): y[r] = x[r] where mask[r] != 0, else zero bits.
template <typename V>
__global__ void __launch_bounds__(kThreads) mask_rows_kernel(const V* __restrict__ x,
                                                             const uint8_t* __restrict__ mask,
                                                             V* __restrict__ y, int64_t rows,
                                                             int64_t per_row) {
  const int64_t total = rows * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t r = i / per_row;
    V v{};
    if (mask[r]) v = x[i];
    y[i] = v;
  }
}

// Masked residual add (model.py:199 `mask(r + down(f))`): y[r, :] = a[r, :] + b[r, :]
// in FP32 (b promoted exactly) where mask[r] != 0, else zero; a and y FP32. Four
// elements per thread (width % 4 == 0, 16/8-byte aligned rows).
template <typename TB>
__global__ void __launch_bounds__(kThreads) masked_add_kernel(const float* __restrict__ a, const TB* __restrict__ b,
                                                              const uint8_t* __restrict__ mask, float* __restrict__ y,
                                                              int64_t rows, int width) {
  const int quads = width / 4;
  const int64_t total = rows * quads;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t r = i / quads;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (mask[r]) {
      const float4 x = load4(a + 4 * i), z = load4(b + 4 * i);
      v = make_float4(x.x + z.x, x.y + z.y, x.z + z.z, x.w + z.w);
    }
    store4(y + 4 * i, v);
  }
}

__device__ __forceinline__ int64_t clamp_len(int64_t len, int T) {
  return len < 0 ? 0 : (len > T ? T : len);
}

// Valid-prefix reversal (kernels/primitives.py:40-47 `_reverse`;
// kernels/__init__.py:43-54): y[b, t] = x[b, len-1-t] for t < len, else zero.
// Lengths outside [0, T] are clamped to it.
template <typename V>
__global__ void __launch_bounds__(kThreads) reverse_valid_kernel(const V* __restrict__ x,
                                                                 const int64_t* __restrict__ lengths,
                                                                 V* __restrict__ y, int B, int T,
                                                                 int64_t per_row) {
  const int64_t total = static_cast<int64_t>(B) * T * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t c = i % per_row;
    const int64_t bt = i / per_row;
    const int t = static_cast<int>(bt % T);
    const int b = static_cast<int>(bt / T);
    const int64_t len = clamp_len(lengths[b], T);
    V v{};
    if (t < len) v = x[(static_cast<int64_t>(b) * T + (len - 1 - t)) * per_row + c];
    y[i] = v;
  }
}

// Last valid row of every batch entry (decoder.py:63, `mf[arange(b), lengths-1]`):
// y[b] = x[b, len-1]; like PyTorch indexing, len = 0 reads row T-1 (index -1).
template <typename V>
__global__ void __launch_bounds__(kThreads) end_gather_kernel(const V* __restrict__ x,
                                                              const int64_t* __restrict__ lengths,
                                                              V* __restrict__ y, int B, int T,
                                                              int64_t per_row) {
  const int64_t total = static_cast<int64_t>(B) * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int b = static_cast<int>(i / per_row);
    int64_t t = lengths[b] - 1;
    if (t < 0) t += T;
    if (t < 0) t = 0;
    if (t >= T) t = T - 1;
    y[i] = x[(static_cast<int64_t>(b) * T + t) * per_row + i % per_row];
  }
}

int vector_bytes(int64_t row_bytes, const void* x, const void* y) {
  for (int v : {16, 8, 4, 2})
    if (row_bytes % v == 0 && aligned(x, v) && aligned(y, v)) return v;
  return 1;
}

// ---------------------------------------------------------------------------
// SwiGLU (kernels/primitives.py:25-37 `_swiglu`; kernels/__init__.py:30-40):
// y[r, c] = silu(x[r, c]) * x[r, d + c], FP32 math, rounded to the input type.
// ---------------------------------------------------------------------------
template <typename T, bool kVec4>
__global__ void __launch_bounds__(kThreads) swiglu_kernel(const T* __restrict__ x,
                                                          T* __restrict__ y, int64_t rows,
                                                          int d) {
  const int step = kVec4 ? 4 : 1;
  const int64_t per_row = d / step;
  const int64_t total = rows * per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t r = i / per_row;
    const int c = static_cast<int>(i % per_row) * step;
    const T* src = x + r * 2 * d + c;
    T* dst = y + r * d + c;
    if (kVec4) {
      const float4 g = load4(src), u = load4(src + d);
      store4(dst, make_float4(g.x * sigmoid_ieee(g.x) * u.x, g.y * sigmoid_ieee(g.y) * u.y,
                              g.z * sigmoid_ieee(g.z) * u.z, g.w * sigmoid_ieee(g.w) * u.w));
    } else {
      const float g = load_f(src), u = load_f(src + d);
      store_f(dst, g * sigmoid_ieee(g) * u);
    }
  }
}

// ---------------------------------------------------------------------------
// Branch gate (kernels/primitives.py:50-62 `_gate`; kernels/__init__.py:57-81):
// x = [..., 3 * d] split in three branches, y[..., j, :] = x[..., j, :] * 2 sigmoid(g[..., j]).
// ---------------------------------------------------------------------------
template <typename T, typename TG, bool kVec4>
__global__ void __launch_bounds__(kThreads) gated_concat_kernel(const T* __restrict__ x,
                                                                const TG* __restrict__ gate,
                                                                T* __restrict__ y, int64_t rows,
                                                                int d) {
  const int step = kVec4 ? 4 : 1;
  const int64_t per_branch = d / step;
  const int64_t total = rows * 3 * per_branch;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t branch_row = i / per_branch;  // r * 3 + j
    const int c = static_cast<int>(i % per_branch) * step;
    const float s = 2.f * sigmoid_ieee(load_f(gate + branch_row));
    const int64_t off = branch_row * d + c;
    if (kVec4) {
      const float4 v = load4(x + off);
      store4(y + off, make_float4(v.x * s, v.y * s, v.z * s, v.w * s));
    } else {
      store_f(y + off, load_f(x + off) * s);
    }
  }
}

// ---------------------------------------------------------------------------
// Pool4 (kernels/primitives.py:90-113 `_pool4` forward; masking.py:59-69):
// y[b, g] = (sum of x[b, 4g + k] over k < 4 with 4g + k < len) / max(min(len - 4g, 4), 1).
// The sum runs in the reference's order (k = 0..3, FP32) and the divide is
// IEEE, so the result equals the reference kernel's bit for bit.
// ---------------------------------------------------------------------------
template <typename T, typename TY = T>
__global__ void __launch_bounds__(kThreads) pool4_kernel(const T* __restrict__ x,
                                                         const int64_t* __restrict__ lengths,
                                                         TY* __restrict__ y, int B, int T_, int LT,
                                                         int D) {
  const int64_t total = static_cast<int64_t>(B) * LT * D;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int c = static_cast<int>(i % D);
    const int64_t bg = i / D;
    const int g = static_cast<int>(bg % LT);
    const int b = static_cast<int>(bg / LT);
    const int64_t len = clamp_len(lengths[b], T_);
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int64_t src = 4 * static_cast<int64_t>(g) + k;
      if (src < len) acc += load_f(x + (static_cast<int64_t>(b) * T_ + src) * D + c);
    }
    int64_t count = len - 4 * static_cast<int64_t>(g);
    count = count > 4 ? 4 : (count < 1 ? 1 : count);
    store_f(y + i, acc / static_cast<float>(count));
  }
}

// Masked time mean (decoder.py:60-62): y[b, c] = sum_{t < len} x[b, t, c] / len, FP32.
// Sums run in time order in FP32; len = 0 gives 0/0 as the reference does.
template <typename T>
__global__ void __launch_bounds__(kThreads) masked_mean_kernel(const T* __restrict__ x,
                                                               const int64_t* __restrict__ lengths,
                                                               float* __restrict__ y, int B, int T_,
                                                               int D) {
  const int64_t total = static_cast<int64_t>(B) * D;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int c = static_cast<int>(i % D);
    const int b = static_cast<int>(i / D);
    const int64_t raw = lengths[b];
    const int64_t len = clamp_len(raw, T_);
    const T* p = x + static_cast<int64_t>(b) * T_ * D + c;
    float acc = 0.f;
    for (int64_t t = 0; t < len; ++t) acc += load_f(p + t * D);
    y[i] = acc / static_cast<float>(raw);
  }
}

// Depthwise Conv1d over time on [B, T, C] rows (kernels/primitives.py:73-87
// `_dw_forward`, kernels/buffers.py:13-32 `depthwise_masked`):
//   y[b, t, c] = t < len ? sum_k x[b, t + k - K/2, c] w[c, k] + bias[c] : 0,
// zero padding outside [0, T). Inputs are rounded to BF16 first (the autocast
// type the reference converts to), each product and sum is rounded separately
// as in the reference kernel, and the result is BF16. Four channels per thread.
// kResidual: y = bf16(x + bf16(conv)) instead (model.py:188-189 `v + conv` before the
// merge projection, whose autocast input is that sum rounded to BF16).
// kGlu: x holds [B, T, 2C] rows (the local branch's up projection, model.py:122) and the
// conv input is their GLU, bf16(a * (1 / (1 + e^-g))) with a = x[.., c], g = x[.., C + c]
// (PyTorch's glu on a BF16 tensor: FP32 math, one rounding), so h is never written.
template <typename TI, int K, bool kResidual = false, bool kGlu = false>
__global__ void __launch_bounds__(kThreads) depthwise_kernel(const TI* __restrict__ x,
                                                             const bf16* __restrict__ w,
                                                             const bf16* __restrict__ bias,
                                                             const int64_t* __restrict__ lengths,
                                                             bf16* __restrict__ y, int B, int T, int C) {
  const int64_t pitch = kGlu ? 2 * static_cast<int64_t>(C) : C;
  const int quads = C / 4;
  const int64_t total = static_cast<int64_t>(B) * T * quads;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int c = 4 * static_cast<int>(i % quads);
    const int64_t bt = i / quads;
    const int t = static_cast<int>(bt % T);
    const int b = static_cast<int>(bt / T);
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const bool live = t < clamp_len(lengths[b], T);
    if (live) {
#pragma unroll
      for (int k = 0; k < K; ++k) {
        const int src = t + k - K / 2;
        if (src < 0 || src >= T) continue;
        float4 xv = load4(x + (static_cast<int64_t>(b) * T + src) * pitch + c);
        if constexpr (kGlu) {
          const float4 gv = load4(x + (static_cast<int64_t>(b) * T + src) * pitch + C + c);
          auto glu = [](float a, float g) { return a * (1.f / (1.f + expf(-g))); };
          xv = make_float4(glu(xv.x, gv.x), glu(xv.y, gv.y), glu(xv.z, gv.z), glu(xv.w, gv.w));
        }
        const float xs[4] = {bf16_round(xv.x), bf16_round(xv.y), bf16_round(xv.z), bf16_round(xv.w)};
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(xs[j], __bfloat162float(w[(c + j) * K + k])));
      }
      if (bias) {
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] = __fadd_rn(acc[j], __bfloat162float(bias[c + j]));
      }
    }
    if (kResidual) {
      const float4 xc = load4(x + bt * C + c);
      acc[0] = xc.x + bf16_round(acc[0]);
      acc[1] = xc.y + bf16_round(acc[1]);
      acc[2] = xc.z + bf16_round(acc[2]);
      acc[3] = xc.w + bf16_round(acc[3]);
    }
    store4(y + bt * C + c, make_float4(acc[0], acc[1], acc[2], acc[3]));
  }
}

}  // namespace

template <typename TI, bool kResidual = false, bool kGlu = false>
int launch_depthwise(const void* x, const bf16* w, const bf16* bias, const int64_t* lengths, bf16* y,
                     int B, int T, int C, int K, cudaStream_t s) {
  const int grid = grid_for(static_cast<int64_t>(B) * T * (C / 4), kThreads);
  auto X = static_cast<const TI*>(x);
  switch (K) {
    case 3: depthwise_kernel<TI, 3, kResidual, kGlu><<<grid, kThreads, 0, s>>>(X, w, bias, lengths, y, B, T, C); break;
    case 5: depthwise_kernel<TI, 5, kResidual, kGlu><<<grid, kThreads, 0, s>>>(X, w, bias, lengths, y, B, T, C); break;
    case 7: depthwise_kernel<TI, 7, kResidual, kGlu><<<grid, kThreads, 0, s>>>(X, w, bias, lengths, y, B, T, C); break;
    default: return TF_ERR_ARG;
  }
  return launch_status();
}

int launch_mask_rows(const void* x, const uint8_t* mask, void* y, int64_t rows, int64_t row_bytes,
                     cudaStream_t s) {
  const int vb = vector_bytes(row_bytes, x, y);
  const int64_t per_row = row_bytes / vb;
  const int grid = grid_for(rows * per_row, kThreads);
  switch (vb) {
    case 16: mask_rows_kernel<uint4><<<grid, kThreads, 0, s>>>(static_cast<const uint4*>(x), mask, static_cast<uint4*>(y), rows, per_row); break;
    case 8: mask_rows_kernel<uint2><<<grid, kThreads, 0, s>>>(static_cast<const uint2*>(x), mask, static_cast<uint2*>(y), rows, per_row); break;
    case 4: mask_rows_kernel<uint32_t><<<grid, kThreads, 0, s>>>(static_cast<const uint32_t*>(x), mask, static_cast<uint32_t*>(y), rows, per_row); break;
    case 2: mask_rows_kernel<uint16_t><<<grid, kThreads, 0, s>>>(static_cast<const uint16_t*>(x), mask, static_cast<uint16_t*>(y), rows, per_row); break;
    default: mask_rows_kernel<uint8_t><<<grid, kThreads, 0, s>>>(static_cast<const uint8_t*>(x), mask, static_cast<uint8_t*>(y), rows, per_row); break;
  }
  return launch_status();
}

int launch_reverse_valid(const void* x, const int64_t* lengths, void* y, int B, int T,
                         int64_t row_bytes, cudaStream_t s) {
  const int vb = vector_bytes(row_bytes, x, y);
  const int64_t per_row = row_bytes / vb;
  const int grid = grid_for(static_cast<int64_t>(B) * T * per_row, kThreads);
  switch (vb) {
    case 16: reverse_valid_kernel<uint4><<<grid, kThreads, 0, s>>>(static_cast<const uint4*>(x), lengths, static_cast<uint4*>(y), B, T, per_row); break;
    case 8: reverse_valid_kernel<uint2><<<grid, kThreads, 0, s>>>(static_cast<const uint2*>(x), lengths, static_cast<uint2*>(y), B, T, per_row); break;
    case 4: reverse_valid_kernel<uint32_t><<<grid, kThreads, 0, s>>>(static_cast<const uint32_t*>(x), lengths, static_cast<uint32_t*>(y), B, T, per_row); break;
    case 2: reverse_valid_kernel<uint16_t><<<grid, kThreads, 0, s>>>(static_cast<const uint16_t*>(x), lengths, static_cast<uint16_t*>(y), B, T, per_row); break;
    default: reverse_valid_kernel<uint8_t><<<grid, kThreads, 0, s>>>(static_cast<const uint8_t*>(x), lengths, static_cast<uint8_t*>(y), B, T, per_row); break;
  }
  return launch_status();
}

int launch_end_gather(const void* x, const int64_t* lengths, void* y, int B, int T,
                      int64_t row_bytes, cudaStream_t s) {
  const int vb = vector_bytes(row_bytes, x, y);
  const int64_t per_row = row_bytes / vb;
  const int grid = grid_for(static_cast<int64_t>(B) * per_row, kThreads);
  switch (vb) {
    case 16: end_gather_kernel<uint4><<<grid, kThreads, 0, s>>>(static_cast<const uint4*>(x), lengths, static_cast<uint4*>(y), B, T, per_row); break;
    case 8: end_gather_kernel<uint2><<<grid, kThreads, 0, s>>>(static_cast<const uint2*>(x), lengths, static_cast<uint2*>(y), B, T, per_row); break;
    case 4: end_gather_kernel<uint32_t><<<grid, kThreads, 0, s>>>(static_cast<const uint32_t*>(x), lengths, static_cast<uint32_t*>(y), B, T, per_row); break;
    case 2: end_gather_kernel<uint16_t><<<grid, kThreads, 0, s>>>(static_cast<const uint16_t*>(x), lengths, static_cast<uint16_t*>(y), B, T, per_row); break;
    default: end_gather_kernel<uint8_t><<<grid, kThreads, 0, s>>>(static_cast<const uint8_t*>(x), lengths, static_cast<uint8_t*>(y), B, T, per_row); break;
  }
  return launch_status();
}

template <typename T>
int launch_swiglu(const void* x, void* y, int64_t rows, int d, cudaStream_t s) {
  const bool v4 = d % 4 == 0 && aligned(x, 4 * sizeof(T)) && aligned(y, 4 * sizeof(T));
  const int64_t items = rows * (v4 ? d / 4 : d);
  const int grid = grid_for(items, kThreads);
  if (v4)
    swiglu_kernel<T, true><<<grid, kThreads, 0, s>>>(static_cast<const T*>(x), static_cast<T*>(y), rows, d);
  else
    swiglu_kernel<T, false><<<grid, kThreads, 0, s>>>(static_cast<const T*>(x), static_cast<T*>(y), rows, d);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Branch gate over three separate branch tensors (model.py:185-186
// `s = cat((cn, mn, an))`, `gated_concat(s, gate(s))`): branch j is read from its
// own rows (pitch p_j elements), so the FP32 concatenation is never written.
// Branches 0 and 2 have type T02, branch 1 is FP32; the output is the FP32
// [rows, 3 d] row the concatenated form produces (every branch value promotes to
// FP32 exactly, so the result equals it bit for bit).
// ---------------------------------------------------------------------------
template <typename T02, typename TG, bool kVec4>
__global__ void __launch_bounds__(kThreads) gated_branches_kernel(const T02* __restrict__ x0, int64_t p0,
                                                                  const float* __restrict__ x1, int64_t p1,
                                                                  const T02* __restrict__ x2, int64_t p2,
                                                                  const TG* __restrict__ gate,
                                                                  float* __restrict__ y, int64_t rows, int d) {
  const int step = kVec4 ? 4 : 1;
  const int64_t per_branch = d / step;
  const int64_t total = rows * 3 * per_branch;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(kThreads) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * kThreads) {
    const int64_t branch_row = i / per_branch;  // r * 3 + j
    const int64_t r = branch_row / 3;
    const int j = static_cast<int>(branch_row - r * 3);
    const int c = static_cast<int>(i % per_branch) * step;
    const float s = 2.f * sigmoid_ieee(load_f(gate + branch_row));
    const int64_t off = branch_row * d + c;
    if (kVec4) {
      const float4 v = j == 1 ? load4(x1 + r * p1 + c) : load4((j == 0 ? x0 + r * p0 : x2 + r * p2) + c);
      store4(y + off, make_float4(v.x * s, v.y * s, v.z * s, v.w * s));
    } else {
      const float v = j == 1 ? x1[r * p1 + c] : load_f((j == 0 ? x0 + r * p0 : x2 + r * p2) + c);
      y[off] = v * s;
    }
  }
}

template <typename T02, typename TG>
int launch_gated_branches(const void* x0, int64_t p0, const float* x1, int64_t p1, const void* x2, int64_t p2,
                          const void* g, float* y, int64_t rows, int d, cudaStream_t s) {
  const bool v4 = d % 4 == 0 && p0 % 4 == 0 && p1 % 4 == 0 && p2 % 4 == 0 && aligned(x0, 4 * sizeof(T02)) &&
                  aligned(x1, 16) && aligned(x2, 4 * sizeof(T02)) && aligned(y, 16);
  const int64_t items = rows * 3 * (v4 ? d / 4 : d);
  const int grid = grid_for(items, kThreads);
  auto X0 = static_cast<const T02*>(x0);
  auto X2 = static_cast<const T02*>(x2);
  auto G = static_cast<const TG*>(g);
  if (v4)
    gated_branches_kernel<T02, TG, true><<<grid, kThreads, 0, s>>>(X0, p0, x1, p1, X2, p2, G, y, rows, d);
  else
    gated_branches_kernel<T02, TG, false><<<grid, kThreads, 0, s>>>(X0, p0, x1, p1, X2, p2, G, y, rows, d);
  return launch_status();
}

// ---------------------------------------------------------------------------
// Branch gate with its projection (model.py:185-186: `gate(s)` under BF16 autocast,
// then `gated_concat`, kernels/__init__.py:57-81). One warp per row computes
//   g_j = bf16(sum_k s[r, k] w[j, k] + bias[j])     (j = 0..2; FP32 products and sums)
// from the BF16 gate-input row s (rows every `sp` elements, width 3 d), then writes
//   y[r, j, :] = x_j[r, :] * 2 sigmoid(g_j)          (FP32, [rows, 3 d])
// where branches 0 and 2 are read back from s (the BF16 values the concatenation
// holds) and branch 1 from the FP32 rows x1. The second read of s hits L1. The
// three-output projection would otherwise be a GEMM with N = 3, for which the
// library's kernels are far from the roofline. `g` (optional) receives the gate values.
// Requires d % 4 == 0 and 8-/16-byte aligned rows (checked by the entry point).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(kThreads) gate_branches_kernel(const bf16* __restrict__ s, int64_t sp,
                                                                 const float* __restrict__ x1, int64_t p1,
                                                                 const bf16* __restrict__ w,
                                                                 const bf16* __restrict__ bias,
                                                                 float* __restrict__ y, bf16* __restrict__ g,
                                                                 int64_t rows, int d) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  const int width = 3 * d;
  for (int64_t row = blockIdx.x * (kThreads / 32) + (threadIdx.x >> 5); row < rows; row += warps) {
    const bf16* sr = s + row * sp;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
#pragma unroll 3
    for (int c = lane * 4; c < width; c += 128) {
      const float4 v = load4(sr + c);
      const float4 w0 = load4(w + c), w1 = load4(w + width + c), w2 = load4(w + 2 * width + c);
      a0 = fmaf(v.x, w0.x, a0); a0 = fmaf(v.y, w0.y, a0); a0 = fmaf(v.z, w0.z, a0); a0 = fmaf(v.w, w0.w, a0);
      a1 = fmaf(v.x, w1.x, a1); a1 = fmaf(v.y, w1.y, a1); a1 = fmaf(v.z, w1.z, a1); a1 = fmaf(v.w, w1.w, a1);
      a2 = fmaf(v.x, w2.x, a2); a2 = fmaf(v.y, w2.y, a2); a2 = fmaf(v.z, w2.z, a2); a2 = fmaf(v.w, w2.w, a2);
    }
    a0 = warp_sum(a0);
    a1 = warp_sum(a1);
    a2 = warp_sum(a2);
    if (bias) {
      a0 += __bfloat162float(bias[0]);
      a1 += __bfloat162float(bias[1]);
      a2 += __bfloat162float(bias[2]);
    }
    const float g0 = bf16_round(a0), g1 = bf16_round(a1), g2 = bf16_round(a2);
    const float s0 = 2.f * sigmoid_ieee(g0), s1 = 2.f * sigmoid_ieee(g1), s2 = 2.f * sigmoid_ieee(g2);
    float* yr = y + row * width;
    const float* xr = x1 + row * p1;
#pragma unroll 3
    for (int c = lane * 4; c < width; c += 128) {
      const int j = c / d;  // d % 4 == 0: a 4-vector never straddles two branches
      const float4 v = j == 1 ? load4(xr + (c - d)) : load4(sr + c);
      const float sc = j == 0 ? s0 : (j == 1 ? s1 : s2);
      store4(yr + c, make_float4(v.x * sc, v.y * sc, v.z * sc, v.w * sc));
    }
    if (g && lane < 3) g[row * 3 + lane] = __float2bfloat16_rn(lane == 0 ? g0 : (lane == 1 ? g1 : g2));
  }
}

int launch_gate_branches(const bf16* s, int64_t sp, const float* x1, int64_t p1, const bf16* w, const bf16* bias,
                         float* y, bf16* g, int64_t rows, int d, cudaStream_t st) {
  const int grid = grid_for(rows, kThreads / 32);
  gate_branches_kernel<<<grid, kThreads, 0, st>>>(s, sp, x1, p1, w, bias, y, g, rows, d);
  return launch_status();
}

template <typename T, typename TG>
int launch_gated_concat(const void* x, const void* g, void* y, int64_t rows, int d, cudaStream_t s) {
  const bool v4 = d % 4 == 0 && aligned(x, 4 * sizeof(T)) && aligned(y, 4 * sizeof(T));
  const int64_t items = rows * 3 * (v4 ? d / 4 : d);
  const int grid = grid_for(items, kThreads);
  if (v4)
    gated_concat_kernel<T, TG, true><<<grid, kThreads, 0, s>>>(static_cast<const T*>(x), static_cast<const TG*>(g), static_cast<T*>(y), rows, d);
  else
    gated_concat_kernel<T, TG, false><<<grid, kThreads, 0, s>>>(static_cast<const T*>(x), static_cast<const TG*>(g), static_cast<T*>(y), rows, d);
  return launch_status();
}

}  // namespace tf

// ===========================================================================
// C ABI (declarations and reference citations in include/trifusion_b200.h)
// ===========================================================================
namespace {

bool valid_dtype(int d) { return d == TF_F32 || d == TF_BF16; }

}  // namespace

extern "C" {

int tf_rms_fwd(const void* x, int dtype, const float* w, void* y, int64_t rows, int width,
               float eps, void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(dtype)) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!x || !w || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F32)
    return tf::launch_row_norm<0, float, float, float>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s);
  return tf::launch_row_norm<0, tf::bf16, tf::bf16, tf::bf16>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s);
}

int tf_rms_out_fwd(const void* x, int dtype, const float* w, void* y, int y_dtype, int64_t rows, int width,
                   float eps, void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(dtype) || !valid_dtype(y_dtype)) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!x || !w || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tf::bf16;
  if (dtype == TF_F32 && y_dtype == TF_F32)
    return tf::launch_row_norm<0, float, float, float>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s);
  if (dtype == TF_F32)
    return tf::launch_row_norm<0, float, float, bf16>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s);
  if (y_dtype == TF_F32)
    return tf::launch_row_norm<0, bf16, bf16, float>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s);
  return tf::launch_row_norm<0, bf16, bf16, bf16>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s);
}

int tf_rms_pitched_fwd(const void* x, int dtype, const float* w, void* y, int y_dtype, int64_t y_pitch,
                       void* y2, int64_t y2_pitch, int64_t rows, int width, float eps, void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(dtype) || !valid_dtype(y_dtype)) return TF_ERR_ARG;
  if (y_pitch < width || (y2 && y2_pitch < width)) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!x || !w || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tf::bf16;
  auto Y2 = static_cast<bf16*>(y2);
  if (dtype == TF_F32 && y_dtype == TF_F32)
    return tf::launch_row_norm<0, float, float, float>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s,
                                                       nullptr, y_pitch, Y2, y2_pitch);
  if (dtype == TF_F32)
    return tf::launch_row_norm<0, float, float, bf16>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s,
                                                      nullptr, y_pitch, Y2, y2_pitch);
  if (y_dtype == TF_F32)
    return tf::launch_row_norm<0, bf16, bf16, float>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s,
                                                     nullptr, y_pitch, Y2, y2_pitch);
  return tf::launch_row_norm<0, bf16, bf16, bf16>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s,
                                                  nullptr, y_pitch, Y2, y2_pitch);
}

int tf_add_rms_fwd(const float* x, const void* a, int a_dtype, const float* w, float* sum, void* y, int y_dtype,
                   int64_t rows, int width, float eps, void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(a_dtype) || !valid_dtype(y_dtype)) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!x || !a || !w || !sum || !y) return TF_ERR_ARG;
  if (width % 4 || !tf::aligned(sum, 16)) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tf::bf16;
  if (a_dtype == TF_BF16 && y_dtype == TF_BF16)
    return tf::launch_row_norm<4, float, bf16, bf16>(x, a, nullptr, w, nullptr, y, rows, width, eps, s, sum);
  if (a_dtype == TF_BF16)
    return tf::launch_row_norm<4, float, bf16, float>(x, a, nullptr, w, nullptr, y, rows, width, eps, s, sum);
  if (y_dtype == TF_BF16)
    return tf::launch_row_norm<4, float, float, bf16>(x, a, nullptr, w, nullptr, y, rows, width, eps, s, sum);
  return tf::launch_row_norm<4, float, float, float>(x, a, nullptr, w, nullptr, y, rows, width, eps, s, sum);
}

int tf_rms_silu_fwd(const void* x, int dtype, const float* w, void* y, int64_t rows, int width, float eps,
                    void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(dtype)) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!x || !w || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F32)
    return tf::launch_row_norm<3, float, float, float>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps, s);
  return tf::launch_row_norm<3, tf::bf16, tf::bf16, tf::bf16>(x, nullptr, nullptr, w, nullptr, y, rows, width, eps,
                                                            s);
}

int tf_evidence_norm_out_fwd(const void* x, int x_dtype, const void* value, const void* gate, int vg_dtype,
                             const float* w, const uint8_t* mask, void* y, int y_dtype, int64_t rows, int width,
                             float eps, void* stream) {
  if (y_dtype == TF_F32)
    return tf_evidence_norm_fwd(x, x_dtype, value, gate, vg_dtype, w, mask, static_cast<float*>(y), rows, width, eps,
                                stream);
  if (rows < 0 || width <= 0 || !valid_dtype(x_dtype) || !valid_dtype(vg_dtype) || y_dtype != TF_BF16)
    return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!x || !value || !gate || !w || !mask || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tf::bf16;
  if (x_dtype == TF_F32 && vg_dtype == TF_F32)
    return tf::launch_row_norm<1, float, float, bf16>(x, value, gate, w, mask, y, rows, width, eps, s);
  if (x_dtype == TF_F32)
    return tf::launch_row_norm<1, float, bf16, bf16>(x, value, gate, w, mask, y, rows, width, eps, s);
  if (vg_dtype == TF_F32)
    return tf::launch_row_norm<1, bf16, float, bf16>(x, value, gate, w, mask, y, rows, width, eps, s);
  return tf::launch_row_norm<1, bf16, bf16, bf16>(x, value, gate, w, mask, y, rows, width, eps, s);
}

int tf_evidence_norm_pitched_fwd(const void* x, int x_dtype, const void* value, const void* gate, int vg_dtype,
                                 int64_t vg_pitch, const float* w, const uint8_t* mask, void* y, int y_dtype,
                                 int64_t rows, int width, float eps, void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(x_dtype) || !valid_dtype(vg_dtype) || !valid_dtype(y_dtype))
    return TF_ERR_ARG;
  if (vg_pitch < width) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!x || !value || !gate || !w || !mask || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tf::bf16;
  const int64_t p = vg_pitch;
#define TF_EVIDENCE(TX, TA, TY) \
  tf::launch_row_norm<1, TX, TA, TY>(x, value, gate, w, mask, y, rows, width, eps, s, nullptr, 0, nullptr, 0, p)
  if (y_dtype == TF_F32) {
    if (x_dtype == TF_F32) return vg_dtype == TF_F32 ? TF_EVIDENCE(float, float, float) : TF_EVIDENCE(float, bf16, float);
    return vg_dtype == TF_F32 ? TF_EVIDENCE(bf16, float, float) : TF_EVIDENCE(bf16, bf16, float);
  }
  if (x_dtype == TF_F32) return vg_dtype == TF_F32 ? TF_EVIDENCE(float, float, bf16) : TF_EVIDENCE(float, bf16, bf16);
  return vg_dtype == TF_F32 ? TF_EVIDENCE(bf16, float, bf16) : TF_EVIDENCE(bf16, bf16, bf16);
#undef TF_EVIDENCE
}

int tf_evidence_norm_fwd(const void* x, int x_dtype, const void* value, const void* gate,
                         int vg_dtype, const float* w, const uint8_t* mask, float* y,
                         int64_t rows, int width, float eps, void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(x_dtype) || !valid_dtype(vg_dtype)) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!x || !value || !gate || !w || !mask || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tf::bf16;
  if (x_dtype == TF_F32 && vg_dtype == TF_F32)
    return tf::launch_row_norm<1, float, float, float>(x, value, gate, w, mask, y, rows, width, eps, s);
  if (x_dtype == TF_F32)
    return tf::launch_row_norm<1, float, bf16, float>(x, value, gate, w, mask, y, rows, width, eps, s);
  if (vg_dtype == TF_F32)
    return tf::launch_row_norm<1, bf16, float, float>(x, value, gate, w, mask, y, rows, width, eps, s);
  return tf::launch_row_norm<1, bf16, bf16, float>(x, value, gate, w, mask, y, rows, width, eps, s);
}

int tf_mean_norm_fwd(const void* a, const void* b, int dtype, const float* w, float* y,
                     int64_t rows, int width, float eps, void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(dtype)) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!a || !b || !w || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F32)
    return tf::launch_row_norm<2, float, float, float>(a, b, nullptr, w, nullptr, y, rows, width, eps, s);
  return tf::launch_row_norm<2, tf::bf16, tf::bf16, float>(a, b, nullptr, w, nullptr, y, rows, width, eps, s);
}

int tf_mean_norm_copy_fwd(const void* a, const void* b, int dtype, const float* w, float* y, void* y2,
                          int64_t y2_pitch, int64_t rows, int width, float eps, void* stream) {
  if (rows < 0 || width <= 0 || !valid_dtype(dtype) || y2_pitch < width) return TF_ERR_ARG;
  if (rows == 0) return TF_OK;
  if (!a || !b || !w || !y || !y2) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto Y2 = static_cast<tf::bf16*>(y2);
  if (dtype == TF_F32)
    return tf::launch_row_norm<2, float, float, float>(a, b, nullptr, w, nullptr, y, rows, width, eps, s, nullptr,
                                                       0, Y2, y2_pitch);
  return tf::launch_row_norm<2, tf::bf16, tf::bf16, float>(a, b, nullptr, w, nullptr, y, rows, width, eps, s,
                                                           nullptr, 0, Y2, y2_pitch);
}

int tf_mamba_controls_fwd(const void* a, const void* ddt, int dtype, const int64_t* strides,
                          const float* dt_bias, float a_floor, float* adt, float* dt, int batch,
                          int seqlen, int heads, void* stream) {
  if (batch < 0 || seqlen < 0 || heads < 0 || !valid_dtype(dtype) || !strides) return TF_ERR_ARG;
  if (batch == 0 || seqlen == 0 || heads == 0) return TF_OK;
  if (!a || !ddt || !dt_bias || !adt || !dt) return TF_ERR_ARG;
  if (strides[2] != 1 || strides[5] != 1) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = tf::grid_for(static_cast<int64_t>(batch) * seqlen * heads, tf::kThreads);
  if (dtype == TF_F32)
    tf::controls_kernel<float><<<grid, tf::kThreads, 0, s>>>(
        static_cast<const float*>(a), static_cast<const float*>(ddt), strides[0], strides[1],
        strides[3], strides[4], dt_bias, a_floor, adt, dt, batch, seqlen, heads);
  else
    tf::controls_kernel<tf::bf16><<<grid, tf::kThreads, 0, s>>>(
        static_cast<const tf::bf16*>(a), static_cast<const tf::bf16*>(ddt), strides[0], strides[1],
        strides[3], strides[4], dt_bias, a_floor, adt, dt, batch, seqlen, heads);
  return tf::launch_status();
}

int tf_mask_rows_fwd(const void* x, const uint8_t* mask, void* y, int64_t rows,
                     int64_t row_bytes, void* stream) {
  if (rows < 0 || row_bytes < 0) return TF_ERR_ARG;
  if (rows == 0 || row_bytes == 0) return TF_OK;
  if (!x || !mask || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  return tf::launch_mask_rows(x, mask, y, rows, row_bytes, static_cast<cudaStream_t>(stream));
}

int tf_masked_add_fwd(const float* a, const void* b, int b_dtype, const uint8_t* mask, float* y, int64_t rows,
                      int width, void* stream) {
  if (rows < 0 || width < 0 || !valid_dtype(b_dtype)) return TF_ERR_ARG;
  if (rows == 0 || width == 0) return TF_OK;
  if (!a || !b || !mask || !y) return TF_ERR_ARG;
  if (width % 4 || !tf::aligned(a, 16) || !tf::aligned(y, 16) || !tf::aligned(b, b_dtype == TF_F32 ? 16 : 8))
    return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = tf::grid_for(rows * (width / 4), tf::kThreads);
  if (b_dtype == TF_F32)
    tf::masked_add_kernel<float><<<grid, tf::kThreads, 0, s>>>(a, static_cast<const float*>(b), mask, y, rows, width);
  else
    tf::masked_add_kernel<tf::bf16><<<grid, tf::kThreads, 0, s>>>(a, static_cast<const tf::bf16*>(b), mask, y, rows,
                                                                  width);
  return tf::launch_status();
}

int tf_reverse_valid_fwd(const void* x, const int64_t* lengths, void* y, int batch, int seqlen,
                         int64_t row_bytes, void* stream) {
  if (batch < 0 || seqlen < 0 || row_bytes < 0) return TF_ERR_ARG;
  if (batch == 0 || seqlen == 0 || row_bytes == 0) return TF_OK;
  if (!x || !lengths || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  return tf::launch_reverse_valid(x, lengths, y, batch, seqlen, row_bytes,
                                  static_cast<cudaStream_t>(stream));
}

int tf_swiglu_fwd(const void* x, int dtype, void* y, int64_t rows, int d, void* stream) {
  if (rows < 0 || d < 0 || !valid_dtype(dtype)) return TF_ERR_ARG;
  if (rows == 0 || d == 0) return TF_OK;
  if (!x || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == TF_F32) return tf::launch_swiglu<float>(x, y, rows, d, s);
  return tf::launch_swiglu<tf::bf16>(x, y, rows, d, s);
}

int tf_gated_concat_fwd(const void* x, int dtype, const void* gate, int gate_dtype, void* y,
                        int64_t rows, int d, void* stream) {
  if (rows < 0 || d < 0 || !valid_dtype(dtype) || !valid_dtype(gate_dtype)) return TF_ERR_ARG;
  if (rows == 0 || d == 0) return TF_OK;
  if (!x || !gate || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tf::bf16;
  if (dtype == TF_F32 && gate_dtype == TF_F32) return tf::launch_gated_concat<float, float>(x, gate, y, rows, d, s);
  if (dtype == TF_F32) return tf::launch_gated_concat<float, bf16>(x, gate, y, rows, d, s);
  if (gate_dtype == TF_F32) return tf::launch_gated_concat<bf16, float>(x, gate, y, rows, d, s);
  return tf::launch_gated_concat<bf16, bf16>(x, gate, y, rows, d, s);
}

int tf_gated_branches_fwd(const void* x0, const float* x1, const void* x2, int dtype, const int64_t* pitches,
                          const void* gate, int gate_dtype, float* y, int64_t rows, int d, void* stream) {
  if (rows < 0 || d < 0 || !valid_dtype(dtype) || !valid_dtype(gate_dtype) || !pitches) return TF_ERR_ARG;
  if (pitches[0] < d || pitches[1] < d || pitches[2] < d) return TF_ERR_ARG;
  if (rows == 0 || d == 0) return TF_OK;
  if (!x0 || !x1 || !x2 || !gate || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  using tf::bf16;
  const int64_t p0 = pitches[0], p1 = pitches[1], p2 = pitches[2];
  if (dtype == TF_F32 && gate_dtype == TF_F32)
    return tf::launch_gated_branches<float, float>(x0, p0, x1, p1, x2, p2, gate, y, rows, d, s);
  if (dtype == TF_F32) return tf::launch_gated_branches<float, bf16>(x0, p0, x1, p1, x2, p2, gate, y, rows, d, s);
  if (gate_dtype == TF_F32)
    return tf::launch_gated_branches<bf16, float>(x0, p0, x1, p1, x2, p2, gate, y, rows, d, s);
  return tf::launch_gated_branches<bf16, bf16>(x0, p0, x1, p1, x2, p2, gate, y, rows, d, s);
}

int tf_gate_branches_fwd(const void* s, int64_t s_pitch, const float* x1, int64_t x1_pitch, const void* w,
                         const void* bias, float* y, void* g, int64_t rows, int d, void* stream) {
  if (rows < 0 || d < 0) return TF_ERR_ARG;
  if (s_pitch < 3 * static_cast<int64_t>(d) || x1_pitch < d) return TF_ERR_ARG;
  if (rows == 0 || d == 0) return TF_OK;
  if (!s || !x1 || !w || !y) return TF_ERR_ARG;
  using tf::aligned;
  if (d % 4 || s_pitch % 4 || x1_pitch % 4 || !aligned(s, 8) || !aligned(w, 8) || !aligned(x1, 16) ||
      !aligned(y, 16))
    return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  using tf::bf16;
  return tf::launch_gate_branches(static_cast<const bf16*>(s), s_pitch, x1, x1_pitch, static_cast<const bf16*>(w),
                                  static_cast<const bf16*>(bias), y, static_cast<bf16*>(g), rows, d,
                                  static_cast<cudaStream_t>(stream));
}

int tf_pool4_fwd(const void* x, int dtype, const int64_t* lengths, void* y, int batch, int seqlen,
                 int width, void* stream) {
  if (batch < 0 || seqlen < 0 || width < 0 || !valid_dtype(dtype)) return TF_ERR_ARG;
  if (batch == 0 || seqlen == 0 || width == 0) return TF_OK;
  if (!x || !lengths || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int lt = (seqlen + 3) / 4;
  const int grid = tf::grid_for(static_cast<int64_t>(batch) * lt * width, tf::kThreads);
  if (dtype == TF_F32)
    tf::pool4_kernel<float><<<grid, tf::kThreads, 0, s>>>(static_cast<const float*>(x), lengths,
                                                          static_cast<float*>(y), batch, seqlen, lt, width);
  else
    tf::pool4_kernel<tf::bf16><<<grid, tf::kThreads, 0, s>>>(static_cast<const tf::bf16*>(x), lengths,
                                                             static_cast<tf::bf16*>(y), batch, seqlen, lt, width);
  return tf::launch_status();
}

int tf_pool4_out_fwd(const void* x, int dtype, const int64_t* lengths, void* y, int y_dtype, int batch, int seqlen,
                     int width, void* stream) {
  if (y_dtype == dtype) return tf_pool4_fwd(x, dtype, lengths, y, batch, seqlen, width, stream);
  if (batch < 0 || seqlen < 0 || width < 0 || dtype != TF_F32 || y_dtype != TF_BF16) return TF_ERR_ARG;
  if (batch == 0 || seqlen == 0 || width == 0) return TF_OK;
  if (!x || !lengths || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const int lt = (seqlen + 3) / 4;
  const int grid = tf::grid_for(static_cast<int64_t>(batch) * lt * width, tf::kThreads);
  tf::pool4_kernel<float, tf::bf16><<<grid, tf::kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const float*>(x), lengths, static_cast<tf::bf16*>(y), batch, seqlen, lt, width);
  return tf::launch_status();
}

int tf_masked_mean_fwd(const void* x, int dtype, const int64_t* lengths, float* y, int batch,
                       int seqlen, int width, void* stream) {
  if (batch < 0 || seqlen < 0 || width < 0 || !valid_dtype(dtype)) return TF_ERR_ARG;
  if (batch == 0 || width == 0) return TF_OK;
  if (!x || !lengths || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int grid = tf::grid_for(static_cast<int64_t>(batch) * width, tf::kThreads);
  if (dtype == TF_F32)
    tf::masked_mean_kernel<float><<<grid, tf::kThreads, 0, s>>>(static_cast<const float*>(x), lengths, y,
                                                                batch, seqlen, width);
  else
    tf::masked_mean_kernel<tf::bf16><<<grid, tf::kThreads, 0, s>>>(static_cast<const tf::bf16*>(x), lengths,
                                                                   y, batch, seqlen, width);
  return tf::launch_status();
}

int tf_depthwise_masked_fwd(const void* x, int dtype, const void* w, const void* bias,
                            const int64_t* lengths, void* y, int batch, int seqlen, int channels,
                            int taps, void* stream) {
  if (batch < 0 || seqlen < 0 || channels < 0 || !valid_dtype(dtype)) return TF_ERR_ARG;
  if (taps != 3 && taps != 5 && taps != 7) return TF_ERR_ARG;
  if (channels % 4) return TF_ERR_LAYOUT;
  if (batch == 0 || seqlen == 0 || channels == 0) return TF_OK;
  if (!x || !w || !lengths || !y) return TF_ERR_ARG;
  const uintptr_t align = dtype == TF_F32 ? 16 : 8;
  if (reinterpret_cast<uintptr_t>(x) % align || reinterpret_cast<uintptr_t>(y) % 8) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto W = static_cast<const tf::bf16*>(w);
  auto Bs = static_cast<const tf::bf16*>(bias);
  auto Y = static_cast<tf::bf16*>(y);
  if (dtype == TF_F32) return tf::launch_depthwise<float>(x, W, Bs, lengths, Y, batch, seqlen, channels, taps, s);
  return tf::launch_depthwise<tf::bf16>(x, W, Bs, lengths, Y, batch, seqlen, channels, taps, s);
}

int tf_depthwise_residual_fwd(const void* x, int dtype, const void* w, const void* bias, const int64_t* lengths,
                              void* y, int batch, int seqlen, int channels, int taps, void* stream) {
  if (batch < 0 || seqlen < 0 || channels < 0 || !valid_dtype(dtype)) return TF_ERR_ARG;
  if (taps != 3 && taps != 5 && taps != 7) return TF_ERR_ARG;
  if (channels % 4) return TF_ERR_LAYOUT;
  if (batch == 0 || seqlen == 0 || channels == 0) return TF_OK;
  if (!x || !w || !lengths || !y) return TF_ERR_ARG;
  const uintptr_t align = dtype == TF_F32 ? 16 : 8;
  if (reinterpret_cast<uintptr_t>(x) % align || reinterpret_cast<uintptr_t>(y) % 8) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto W = static_cast<const tf::bf16*>(w);
  auto Bs = static_cast<const tf::bf16*>(bias);
  auto Y = static_cast<tf::bf16*>(y);
  if (dtype == TF_F32)
    return tf::launch_depthwise<float, true>(x, W, Bs, lengths, Y, batch, seqlen, channels, taps, s);
  return tf::launch_depthwise<tf::bf16, true>(x, W, Bs, lengths, Y, batch, seqlen, channels, taps, s);
}

int tf_glu_depthwise_fwd(const void* x, const void* w, const void* bias, const int64_t* lengths, void* y,
                         int batch, int seqlen, int channels, int taps, void* stream) {
  if (batch < 0 || seqlen < 0 || channels < 0) return TF_ERR_ARG;
  if (taps != 3 && taps != 5 && taps != 7) return TF_ERR_ARG;
  if (channels % 4) return TF_ERR_LAYOUT;
  if (batch == 0 || seqlen == 0 || channels == 0) return TF_OK;
  if (!x || !w || !lengths || !y) return TF_ERR_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 8 || reinterpret_cast<uintptr_t>(y) % 8) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  return tf::launch_depthwise<tf::bf16, false, true>(x, static_cast<const tf::bf16*>(w),
                                                     static_cast<const tf::bf16*>(bias), lengths,
                                                     static_cast<tf::bf16*>(y), batch, seqlen, channels, taps,
                                                     static_cast<cudaStream_t>(stream));
}

int tf_end_gather_fwd(const void* x, const int64_t* lengths, void* y, int batch, int seqlen,
                      int64_t row_bytes, void* stream) {
  if (batch < 0 || seqlen <= 0 || row_bytes < 0) return batch == 0 ? TF_OK : TF_ERR_ARG;
  if (batch == 0 || row_bytes == 0) return TF_OK;
  if (!x || !lengths || !y) return TF_ERR_ARG;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  return tf::launch_end_gather(x, lengths, y, batch, seqlen, row_bytes,
                               static_cast<cudaStream_t>(stream));
}

}  // extern "C"

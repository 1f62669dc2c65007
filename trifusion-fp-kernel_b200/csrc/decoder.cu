// Decoder query read (decoder.py:24-30 `QueryRead.forward`, attention.py:8-18):
// 10 learned queries x 8 heads of width 32 attend, in FP32, over one clip's keys,
//   h[b, i, 32 c + d] = sum_j softmax_j(q_c[i] . k_c[b, j] / sqrt(32)) v_c[b, j, d],
// keys j valid when j < min(T, lengths[b] * keys_per_length) (the bool mask of the
// reference: `grids.mask` for the deep read, the 8-band expansion of the fine mask
// for the fine read). q, k and v are the BF16 projection outputs, widened to FP32
// exactly as the reference's `.float()` does; the result is rounded once to BF16.
//
// Split over keys (the key count is far larger than the query count, and one
// (batch, head) pair per CTA leaves most SMs idle): each CTA takes kSplit keys of
// one (batch, head), stages their k and v rows, and writes the split's FP32
// softmax state (max, sum, unnormalised output); a merge pass rescales the splits
// to the common max and divides. k and v are read straight from the [B, T, 512]
// projection rows (k of head c at columns 32 c, v at 256 + 32 c), so neither the
// reference's permute nor its FP32 copies are made, and the output is written in
// the [B, 10, 256] row layout the out projection reads.
#include <cstdint>

#include "../../include/trifusion_b200.h"
#include "tf_common.cuh"
#include "tf_host.cuh"

namespace tf {
namespace {

constexpr int kQueries = 10;
constexpr int kHeads = 8;
constexpr int kWidth = 32;
constexpr int kSplit = 256;    // keys per CTA
constexpr int kThreads = 128;  // two keys per thread
constexpr int kState = kWidth + 2;  // per query and split: output[32], max, sum

__device__ __forceinline__ void bf16x8_to_f(const uint4 u, float* f) {
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}

__global__ void __launch_bounds__(kThreads) query_read_split_kernel(const bf16* __restrict__ q,
                                                                    const bf16* __restrict__ kv, int64_t pitch,
                                                                    const int64_t* __restrict__ lengths,
                                                                    int keys_per_length, int T, int splits,
                                                                    float scale, float* __restrict__ state) {
  __shared__ float qs[kQueries][kWidth];
  __shared__ float ps[kQueries][kSplit];
  __shared__ float vs[kSplit][kWidth + 1];
  const int split = blockIdx.x, head = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  int64_t valid = lengths[b] * static_cast<int64_t>(keys_per_length);
  if (valid > T) valid = T;
  if (valid < 0) valid = 0;
  const int64_t first = static_cast<int64_t>(split) * kSplit;
  float* out = state + ((static_cast<int64_t>(b) * kHeads + head) * splits + split) * kQueries * kState;
  if (first >= valid) {  // every key of this split is masked
    for (int e = tid; e < kQueries * kState; e += kThreads) {
      const int r = e % kState;
      out[e] = r == kWidth ? -INFINITY : 0.f;
    }
    return;
  }
  for (int e = tid; e < kQueries * kWidth; e += kThreads) {
    const int i = e / kWidth, d = e % kWidth;
    qs[i][d] = __bfloat162float(q[i * (kHeads * kWidth) + head * kWidth + d]);
  }
  __syncthreads();
  // Scores of this thread's two keys for all queries; v rows into shared memory.
#pragma unroll 1
  for (int jj = 0; jj < 2; ++jj) {
    const int j = tid + jj * kThreads;
    const int64_t key = first + j;
    float kf[kWidth], vf[kWidth];
    if (key < valid) {
      const bf16* row = kv + (static_cast<int64_t>(b) * T + key) * pitch;
      const uint4* kr = reinterpret_cast<const uint4*>(row + head * kWidth);
      const uint4* vr = reinterpret_cast<const uint4*>(row + kHeads * kWidth + head * kWidth);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        bf16x8_to_f(__ldg(kr + c), kf + 8 * c);
        bf16x8_to_f(__ldg(vr + c), vf + 8 * c);
      }
#pragma unroll
      for (int i = 0; i < kQueries; ++i) {
        float s = 0.f;
#pragma unroll
        for (int d = 0; d < kWidth; ++d) s = fmaf(qs[i][d], kf[d], s);
        ps[i][j] = s * scale;
      }
    } else {
#pragma unroll
      for (int d = 0; d < kWidth; ++d) vf[d] = 0.f;
#pragma unroll
      for (int i = 0; i < kQueries; ++i) ps[i][j] = -INFINITY;
    }
#pragma unroll
    for (int d = 0; d < kWidth; ++d) vs[j][d] = vf[d];
  }
  __syncthreads();
  // Softmax state per query: warp w takes queries w, w + 4, w + 8.
  const int warp = tid >> 5, lane = tid & 31;
  for (int i = warp; i < kQueries; i += kThreads / 32) {
    float m = -INFINITY;
    for (int j = lane; j < kSplit; j += 32) m = fmaxf(m, ps[i][j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int j = lane; j < kSplit; j += 32) {
      const float s = ps[i][j];
      const float p = s == -INFINITY ? 0.f : expf(s - m);
      ps[i][j] = p;
      l += p;
    }
    l = warp_sum(l);
    if (lane == 0) {
      out[i * kState + kWidth] = m;
      out[i * kState + kWidth + 1] = l;
    }
  }
  __syncthreads();
  // Unnormalised output: sum_j p[i, j] v[j, d], one (query, column) per thread.
  for (int e = tid; e < kQueries * kWidth; e += kThreads) {
    const int i = e / kWidth, d = e % kWidth;
    float acc = 0.f;
#pragma unroll 8
    for (int j = 0; j < kSplit; ++j) acc = fmaf(ps[i][j], vs[j][d], acc);
    out[i * kState + d] = acc;
  }
}

// Merge the splits of one (batch, head): y = sum_s o_s e^(m_s - M) / sum_s l_s e^(m_s - M).
__global__ void __launch_bounds__(kQueries * kWidth) query_read_merge_kernel(const float* __restrict__ state,
                                                                             int splits, bf16* __restrict__ y) {
  const int head = blockIdx.x, b = blockIdx.y;
  const int i = threadIdx.x / kWidth, d = threadIdx.x % kWidth;
  const float* st = state + (static_cast<int64_t>(b) * kHeads + head) * splits * kQueries * kState + i * kState;
  float m = -INFINITY;
  for (int s = 0; s < splits; ++s) m = fmaxf(m, st[s * kQueries * kState + kWidth]);
  float l = 0.f, o = 0.f;
  if (m != -INFINITY) {
    for (int s = 0; s < splits; ++s) {
      const float* x = st + s * kQueries * kState;
      const float ms = x[kWidth];
      if (ms == -INFINITY) continue;
      const float f = expf(ms - m);
      l = fmaf(x[kWidth + 1], f, l);
      o = fmaf(x[d], f, o);
    }
  }
  // No valid key at all: the reference's softmax over an all-masked row is NaN.
  const float r = l > 0.f ? o / l : __int_as_float(0x7fc00000);
  y[(static_cast<int64_t>(b) * kQueries + i) * (kHeads * kWidth) + head * kWidth + d] = __float2bfloat16_rn(r);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Local evidence (decoder.py:65-76): per clip b and class c, the scores
// s_t = float(local[b, t, c]) (-inf where t >= fine_lengths[b]), the k = min(25, T)
// largest of them (torch.topk: sorted, largest first), and the masked mean of the
// chosen frames' BF16 feature rows,
//   top[b, c, :] = sum_r valid_r * float(features[b, idx_r, :]) / sum_r valid_r,
// valid_r = r < min(fine_lengths[b], k). The unmasked FP32 copy of the logits
// (`local.float()`, a decoder output) is written on the way.
//
// Selection: each score maps to an order-preserving 32-bit key (NaN largest, as
// topk orders it); a four-pass 8-bit radix select finds the k-th largest key K; the
// keys above K and then the lowest-indexed keys equal to K are taken, and the k
// picks are ranked by (key descending, index ascending). Ties at K therefore
// resolve to the earliest frames.
// ---------------------------------------------------------------------------
constexpr int kTopThreads = 256;
constexpr int kTopMax = 25;       // decoder.py:69 `min(25, tf)`
constexpr int kFeature = 256;     // local_features width
constexpr int kTopMaxTime = 12288;  // frames held in shared memory (48 KB of keys)

__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  if (f != f) return 0xffffffffu;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Masked mean of the chosen rows, in rank order; invalid ranks add 0 * x. All k rows
// are loaded before the sum, so their latencies overlap.
__device__ __forceinline__ void topk_mean(const bf16* __restrict__ features, int64_t feat_pitch, int b, int c,
                                          int T, int k, int valid, const int* sorted_idx, float* __restrict__ top) {
  const int count = valid < k ? valid : k;
  for (int j = threadIdx.x; j < kFeature; j += kTopThreads) {
    float xr[kTopMax];
#pragma unroll
    for (int r = 0; r < kTopMax; ++r)
      xr[r] = r < k ? bf2f(features[(static_cast<int64_t>(b) * T + sorted_idx[r]) * feat_pitch + j]) : 0.f;
    float acc = 0.f;
#pragma unroll
    for (int r = 0; r < kTopMax; ++r)
      if (r < k) acc += xr[r] * (r < count ? 1.f : 0.f);
    top[(static_cast<int64_t>(b) * 2 + c) * kFeature + j] = acc / static_cast<float>(count);
  }
}

__global__ void __launch_bounds__(kTopThreads) local_topk_kernel(const bf16* __restrict__ local, int64_t local_pitch,
                                                                 const bf16* __restrict__ features,
                                                                 int64_t feat_pitch,
                                                                 const int64_t* __restrict__ fine_lengths, int T,
                                                                 int k, float* __restrict__ local_f32,
                                                                 float* __restrict__ top) {
  extern __shared__ uint32_t keys[];  // [T]
  __shared__ int hist[256];
  __shared__ int picks[kTopMax];
  __shared__ int sorted_idx[kTopMax];
  __shared__ int ctl[4];  // digit, remaining, greater count, equal count
  const int c = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  int64_t len = fine_lengths[b];
  const int valid = static_cast<int>(len < 0 ? 0 : (len > T ? T : len));
  const uint32_t masked_key = order_key(-INFINITY);
  for (int t = tid; t < T; t += kTopThreads) {
    const int64_t row = static_cast<int64_t>(b) * T + t;
    const float v = bf2f(local[row * local_pitch + c]);
    local_f32[row * 2 + c] = v;
    keys[t] = t < valid ? order_key(v) : masked_key;
  }
  // Radix select of the k-th largest key, 8 bits at a time from the top.
  uint32_t prefix = 0, pmask = 0;
  int remaining = k;
  for (int pass = 0; pass < 4 && k > 0; ++pass) {
    const int shift = 24 - 8 * pass;
    hist[tid] = 0;
    __syncthreads();  // also orders the key stores before the first pass
    for (int t = tid; t < T; t += kTopThreads) {
      const uint32_t key = keys[t];
      if ((key & pmask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1);
    }
    __syncthreads();
    if (warp == 0) {
      // Lane l sums bins 255-8l down to 248-8l; an exclusive scan from the top then
      // finds the bin where the count of larger keys first reaches `remaining`.
      int part = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) part += hist[255 - 8 * lane - i];
      int incl = part;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += n;
      }
      const int excl = incl - part;
      const bool here = excl < remaining && incl >= remaining;
      if (here) {
        int above = excl;
        for (int i = 0; i < 8; ++i) {
          const int bin = 255 - 8 * lane - i;
          const int h = hist[bin];
          if (above + h >= remaining) {
            ctl[0] = bin;
            ctl[1] = remaining - above;
            break;
          }
          above += h;
        }
      }
    }
    __syncthreads();
    prefix |= static_cast<uint32_t>(ctl[0]) << shift;
    pmask |= 0xffu << shift;
    remaining = ctl[1];
    __syncthreads();  // every thread has read ctl before the next pass rewrites it
  }
  // Picks: every key above the k-th, then the earliest `remaining` keys equal to it.
  if (tid == 0) ctl[2] = 0;
  __syncthreads();
  for (int t = tid; t < T && k > 0; t += kTopThreads)
    if (keys[t] > prefix) picks[atomicAdd(&ctl[2], 1)] = t;
  __syncthreads();
  const int greater = ctl[2];
  if (warp == 0 && k > 0) {
    int taken = 0;
    for (int t0 = 0; t0 < T && taken < remaining; t0 += 32) {
      const int t = t0 + lane;
      const bool eq = t < T && keys[t] == prefix;
      const uint32_t bal = __ballot_sync(0xffffffffu, eq);
      const int pos = taken + __popc(bal & ((1u << lane) - 1u));
      if (eq && pos < remaining) picks[greater + pos] = t;
      taken += __popc(bal);
    }
  }
  __syncthreads();
  if (tid < k) {
    const int ti = picks[tid];
    const uint32_t ki = keys[ti];
    int rank = 0;
    for (int j = 0; j < k; ++j) {
      const int tj = picks[j];
      const uint32_t kj = keys[tj];
      rank += (kj > ki) || (kj == ki && tj < ti);
    }
    sorted_idx[rank] = ti;
  }
  __syncthreads();
  topk_mean(features, feat_pitch, b, c, T, k, valid, sorted_idx, top);
}

// ---------------------------------------------------------------------------
// Decoder heads (decoder.py:77-89) as three launches:
//  1. voice = silu(voice_lat(cat(deep_q[0], fine_q[0], global, top[:, 0], memory))) and
//     music likewise with the group-1 reads and top[:, 1];
//  2. file hidden = silu(file_head[0](cat(deep_q[2], fine_q[2], global, memory, voice, music)));
//  3. v = voice_head(voice), m = music_head(music), f = file_head[2](file hidden),
//     logits = [f, v0, m0, v1, m1] in FP32.
// deep_q[g] / fine_q[g] are the group means of the query-read rows h [B, 10, 256]
// (rows 0-3, 4-7, 8-9): FP32 sums rounded once to BF16 (torch's mean of BF16). Every
// concatenated input is what autocast hands the projection: FP32 parts (top) rounded
// to BF16, BF16 parts as they are. A projection is a BF16 x BF16 product accumulated
// in FP32, plus the BF16 bias, rounded to BF16; SiLU acts on that BF16 value and
// rounds again (torch's silu on a BF16 tensor). Only the FP32 summation order
// differs from cuBLAS.
// ---------------------------------------------------------------------------
constexpr int kHeadWidth = 256;   // every hidden layer and input part is 256 wide
constexpr int kHeadRows = 8;      // batch rows per CTA
constexpr int kHeadCols = 8;      // output columns per CTA (one per warp)
constexpr int kHeadThreads = 256;
constexpr int kHeadMaxParts = 6;

struct HeadPart {
  const void* ptr;       // row b at ptr + b * batch_stride elements
  int64_t batch_stride;
  int dtype;             // TF_BF16 or TF_F32
  int rows;              // 1, or the count of consecutive 256-wide rows averaged
};
struct HeadLayer {
  HeadPart part[kHeadMaxParts];
  int nparts;
  const bf16* w;     // [256, nparts * 256]
  const bf16* bias;  // [256]
  bf16* out;         // [batch, 256]
};
struct HeadLayers {
  HeadLayer layer[2];
};

// Raw 16-byte loads of one 8-feature chunk of part `pt` for batch row b (chunk q):
// `rows` loads for BF16 parts (the rows averaged), two for an FP32 part.
__device__ __forceinline__ void head_chunk_load(const HeadPart& pt, int b, int q, uint4 (&raw)[4]) {
  if (pt.dtype == TF_F32) {
    const float* x = static_cast<const float*>(pt.ptr) + b * pt.batch_stride + 8 * q;
    raw[0] = *reinterpret_cast<const uint4*>(x);
    raw[1] = *reinterpret_cast<const uint4*>(x + 4);
    return;
  }
  const bf16* x = static_cast<const bf16*>(pt.ptr) + b * pt.batch_stride + 8 * q;
#pragma unroll
  for (int r = 0; r < 4; ++r)
    if (r < pt.rows) raw[r] = *reinterpret_cast<const uint4*>(x + r * kHeadWidth);
}
// The chunk's 8 values as the projection reads them (see above).
__device__ __forceinline__ void head_chunk_values(const HeadPart& pt, const uint4 (&raw)[4], float (&v)[8]) {
  if (pt.dtype == TF_F32) {
    const float* f = reinterpret_cast<const float*>(raw);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = bf16_round(f[e]);
    return;
  }
  bf16x8_to_f(raw[0], v);
  if (pt.rows == 1) return;
#pragma unroll
  for (int r = 1; r < 4; ++r) {
    if (r < pt.rows) {
      float w[8];
      bf16x8_to_f(raw[r], w);
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] += w[e];
    }
  }
  const float inv = static_cast<float>(pt.rows);
#pragma unroll
  for (int e = 0; e < 8; ++e) v[e] = bf16_round(v[e] / inv);
}

// grid (256 / kHeadCols, ceil(batch / kHeadRows), layers), every layer of the launch
// with kParts parts; dynamic shared memory kHeadRows * kParts * 256 floats (the CTA's
// input rows).
template <int kParts>
__global__ void __launch_bounds__(kHeadThreads) head_layer_kernel(const __grid_constant__ HeadLayers L, int batch) {
  extern __shared__ __align__(16) float xs[];  // [kHeadRows][K]
  constexpr int K = kParts * kHeadWidth;
  constexpr int kChunks = kHeadRows * kParts * (kHeadWidth / 8);
  constexpr int kPerThread = (kChunks + kHeadThreads - 1) / kHeadThreads;
  const HeadLayer& ly = L.layer[blockIdx.z];
  const int row0 = blockIdx.y * kHeadRows;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The warp's weight row (one output column) and every load of the thread's input
  // chunks are issued before any is used.
  const int col = blockIdx.x * kHeadCols + warp;
  const bf16* wrow = ly.w + static_cast<int64_t>(col) * K;
  uint4 wv[kParts];
#pragma unroll
  for (int it = 0; it < kParts; ++it) wv[it] = *reinterpret_cast<const uint4*>(wrow + it * 256 + 8 * lane);
  uint4 raw[kPerThread][4];
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const int e = tid + j * kHeadThreads;
    const int r = e / (kParts * 32), pq = e % (kParts * 32);
    if (e < kChunks && row0 + r < batch) head_chunk_load(ly.part[pq / 32], row0 + r, pq % 32, raw[j]);
  }
#pragma unroll
  for (int j = 0; j < kPerThread; ++j) {
    const int e = tid + j * kHeadThreads;
    if (e >= kChunks) continue;
    const int r = e / (kParts * 32), pq = e % (kParts * 32);
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (row0 + r < batch) head_chunk_values(ly.part[pq / 32], raw[j], v);
    float* dst = xs + r * K + 8 * pq;
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(dst + 4) = make_float4(v[4], v[5], v[6], v[7]);
  }
  __syncthreads();
  float acc[kHeadRows];
#pragma unroll
  for (int r = 0; r < kHeadRows; ++r) acc[r] = 0.f;
#pragma unroll
  for (int it = 0; it < kParts; ++it) {
    const int k0 = it * 256 + 8 * lane;
    float wf[8];
    bf16x8_to_f(wv[it], wf);
#pragma unroll
    for (int r = 0; r < kHeadRows; ++r) {
      const float4 a = *reinterpret_cast<const float4*>(xs + r * K + k0);
      const float4 c = *reinterpret_cast<const float4*>(xs + r * K + k0 + 4);
      const float xv[8] = {a.x, a.y, a.z, a.w, c.x, c.y, c.z, c.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[r] = fmaf(wf[e], xv[e], acc[r]);
    }
  }
#pragma unroll
  for (int r = 0; r < kHeadRows; ++r)
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
  // Lane r stores row row0 + r.
  float v = 0.f;
#pragma unroll
  for (int r = 0; r < kHeadRows; ++r)
    if (lane == r) v = acc[r];
  const int b = row0 + lane;
  if (lane < kHeadRows && b < batch) {
    const float a = bf16_round(v + bf2f(ly.bias[col]));
    ly.out[static_cast<int64_t>(b) * kHeadWidth + col] = __float2bfloat16_rn(a / (1.f + expf(-a)));
  }
}

// One warp per batch row: the three small heads and the logits row.
__global__ void __launch_bounds__(128) head_logits_kernel(const bf16* __restrict__ voice,
                                                          const bf16* __restrict__ music,
                                                          const bf16* __restrict__ fileh,
                                                          const bf16* __restrict__ w_v, const bf16* __restrict__ b_v,
                                                          const bf16* __restrict__ w_m, const bf16* __restrict__ b_m,
                                                          const bf16* __restrict__ w_f, const bf16* __restrict__ b_f,
                                                          float* __restrict__ logits, int batch) {
  const int b = blockIdx.x * 4 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (b >= batch) return;
  auto dot = [&](const bf16* x, const bf16* w) {
    float xf[8], wf[8];
    bf16x8_to_f(*reinterpret_cast<const uint4*>(x + 8 * lane), xf);
    bf16x8_to_f(*reinterpret_cast<const uint4*>(w + 8 * lane), wf);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) s = fmaf(wf[e], xf[e], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
  };
  const bf16* vr = voice + static_cast<int64_t>(b) * kHeadWidth;
  const bf16* mr = music + static_cast<int64_t>(b) * kHeadWidth;
  const bf16* fr = fileh + static_cast<int64_t>(b) * kHeadWidth;
  const float v0 = bf16_round(dot(vr, w_v) + bf2f(b_v[0]));
  const float v1 = bf16_round(dot(vr, w_v + kHeadWidth) + bf2f(b_v[1]));
  const float m0 = bf16_round(dot(mr, w_m) + bf2f(b_m[0]));
  const float m1 = bf16_round(dot(mr, w_m + kHeadWidth) + bf2f(b_m[1]));
  const float f = bf16_round(dot(fr, w_f) + bf2f(b_f[0]));
  if (lane == 0) {
    float* y = logits + static_cast<int64_t>(b) * 5;
    y[0] = f;
    y[1] = v0;
    y[2] = m0;
    y[3] = v1;
    y[4] = m1;
  }
}

}  // namespace
}  // namespace tf

extern "C" {

int64_t tf_query_read_state_floats(int batch, int time) {
  if (batch < 0 || time < 0) return -1;
  const int64_t splits = (time + tf::kSplit - 1) / tf::kSplit;
  return static_cast<int64_t>(batch) * tf::kHeads * splits * tf::kQueries * tf::kState;
}

int tf_query_read_fwd(const void* q, const void* kv, int64_t kv_pitch, const int64_t* lengths, int keys_per_length,
                      float* state, int64_t state_floats, void* y, int batch, int time, void* stream) {
  if (batch < 0 || time < 0 || keys_per_length < 1 || kv_pitch < 2 * tf::kHeads * tf::kWidth) return TF_ERR_ARG;
  if (batch == 0) return TF_OK;
  if (!q || !lengths || !y || (time > 0 && (!kv || !state))) return TF_ERR_ARG;
  if (tf_query_read_state_floats(batch, time) > state_floats && time > 0) return TF_ERR_SIZE;
  if (!tf::aligned16(kv) || kv_pitch % 8) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int splits = (time + tf::kSplit - 1) / tf::kSplit;
  if (splits > 0) {
    const dim3 grid(splits, tf::kHeads, batch);
    tf::query_read_split_kernel<<<grid, tf::kThreads, 0, s>>>(
        static_cast<const tf::bf16*>(q), static_cast<const tf::bf16*>(kv), kv_pitch, lengths, keys_per_length, time,
        splits, 1.f / sqrtf(static_cast<float>(tf::kWidth)), state);
    const int e = tf::launch_status();
    if (e != TF_OK) return e;
  }
  tf::query_read_merge_kernel<<<dim3(tf::kHeads, batch), tf::kQueries * tf::kWidth, 0, s>>>(state, splits,
                                                                                          static_cast<tf::bf16*>(y));
  return tf::launch_status();
}


int tf_local_topk_fwd(const void* local, int64_t local_pitch, const void* features, int64_t feat_pitch,
                      const int64_t* fine_lengths, float* local_f32, float* top, int batch, int time,
                      void* stream) {
  if (batch < 0 || time < 0 || local_pitch < 2 || feat_pitch < tf::kFeature) return TF_ERR_ARG;
  if (batch == 0) return TF_OK;
  if (!fine_lengths || !top || (time > 0 && (!local || !features || !local_f32))) return TF_ERR_ARG;
  if (time > tf::kTopMaxTime) return TF_ERR_SIZE;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const int k = time < tf::kTopMax ? time : tf::kTopMax;
  const size_t smem = static_cast<size_t>(time > 0 ? time : 1) * sizeof(uint32_t);
  if (smem > 32 * 1024)  // beyond the default once the kernel's static arrays are added
    cudaFuncSetAttribute(tf::local_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(tf::kTopMaxTime * sizeof(uint32_t)));
  tf::local_topk_kernel<<<dim3(2, batch), tf::kTopThreads, smem, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const tf::bf16*>(local), local_pitch, static_cast<const tf::bf16*>(features), feat_pitch,
      fine_lengths, time, k, local_f32, top);
  return tf::launch_status();
}

int64_t tf_decoder_heads_scratch_bytes(int batch) {
  if (batch < 0) return -1;
  return static_cast<int64_t>(batch) * 3 * tf::kHeadWidth * 2;
}

int tf_decoder_heads_fwd(const void* deep_rows, const void* fine_rows, const void* global_feature,
                         const void* memory, const float* top, const void* w_voice, const void* b_voice,
                         const void* w_music, const void* b_music, const void* w_vhead, const void* b_vhead,
                         const void* w_mhead, const void* b_mhead, const void* w_file1, const void* b_file1,
                         const void* w_file2, const void* b_file2, void* scratch, int64_t scratch_bytes,
                         float* logits, int batch, void* stream) {
  if (batch < 0) return TF_ERR_ARG;
  if (batch == 0) return TF_OK;
  const void* ptrs[] = {deep_rows, fine_rows, global_feature, memory, top, w_voice, b_voice, w_music, b_music,
                        w_vhead, b_vhead, w_mhead, b_mhead, w_file1, b_file1, w_file2, b_file2, scratch, logits};
  for (const void* p : ptrs)
    if (!p) return TF_ERR_ARG;
  if (scratch_bytes < tf_decoder_heads_scratch_bytes(batch)) return TF_ERR_SIZE;
  const void* vec[] = {deep_rows, fine_rows, global_feature, memory, top,   w_voice, w_music,
                       w_vhead,   w_mhead,   w_file1,        w_file2, scratch};
  for (const void* p : vec)
    if (!tf::aligned16(p)) return TF_ERR_LAYOUT;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  tf::bf16* voice = static_cast<tf::bf16*>(scratch);
  tf::bf16* music = voice + static_cast<int64_t>(batch) * tf::kHeadWidth;
  tf::bf16* fileh = music + static_cast<int64_t>(batch) * tf::kHeadWidth;
  const int64_t rows10 = 10 * tf::kHeadWidth;
  auto part = [](const void* p, int64_t stride, int dtype, int rows) {
    tf::HeadPart h;
    h.ptr = p;
    h.batch_stride = stride;
    h.dtype = dtype;
    h.rows = rows;
    return h;
  };
  const tf::bf16* deep = static_cast<const tf::bf16*>(deep_rows);
  const tf::bf16* fine = static_cast<const tf::bf16*>(fine_rows);
  tf::HeadLayers L = {};
  for (int g = 0; g < 2; ++g) {  // 0: voice (query groups 0-3, top class 0); 1: music (4-7, class 1)
    tf::HeadLayer& ly = L.layer[g];
    ly.part[0] = part(deep + g * 4 * tf::kHeadWidth, rows10, TF_BF16, 4);
    ly.part[1] = part(fine + g * 4 * tf::kHeadWidth, rows10, TF_BF16, 4);
    ly.part[2] = part(global_feature, tf::kHeadWidth, TF_BF16, 1);
    ly.part[3] = part(top + g * tf::kHeadWidth, 2 * tf::kHeadWidth, TF_F32, 1);
    ly.part[4] = part(memory, tf::kHeadWidth, TF_BF16, 1);
    ly.nparts = 5;
    ly.w = static_cast<const tf::bf16*>(g == 0 ? w_voice : w_music);
    ly.bias = static_cast<const tf::bf16*>(g == 0 ? b_voice : b_music);
    ly.out = g == 0 ? voice : music;
  }
  const dim3 grid_lat(tf::kHeadWidth / tf::kHeadCols, (batch + tf::kHeadRows - 1) / tf::kHeadRows, 2);
  tf::head_layer_kernel<5><<<grid_lat, tf::kHeadThreads, tf::kHeadRows * 5 * tf::kHeadWidth * sizeof(float), s>>>(L,
                                                                                                            batch);
  int e = tf::launch_status();
  if (e != TF_OK) return e;
  tf::HeadLayers F = {};
  {
    tf::HeadLayer& ly = F.layer[0];
    ly.part[0] = part(deep + 8 * tf::kHeadWidth, rows10, TF_BF16, 2);
    ly.part[1] = part(fine + 8 * tf::kHeadWidth, rows10, TF_BF16, 2);
    ly.part[2] = part(global_feature, tf::kHeadWidth, TF_BF16, 1);
    ly.part[3] = part(memory, tf::kHeadWidth, TF_BF16, 1);
    ly.part[4] = part(voice, tf::kHeadWidth, TF_BF16, 1);
    ly.part[5] = part(music, tf::kHeadWidth, TF_BF16, 1);
    ly.nparts = 6;
    ly.w = static_cast<const tf::bf16*>(w_file1);
    ly.bias = static_cast<const tf::bf16*>(b_file1);
    ly.out = fileh;
  }
  const dim3 grid_file(tf::kHeadWidth / tf::kHeadCols, (batch + tf::kHeadRows - 1) / tf::kHeadRows, 1);
  tf::head_layer_kernel<6><<<grid_file, tf::kHeadThreads, tf::kHeadRows * 6 * tf::kHeadWidth * sizeof(float), s>>>(
      F, batch);
  e = tf::launch_status();
  if (e != TF_OK) return e;
  tf::head_logits_kernel<<<(batch + 3) / 4, 128, 0, s>>>(
      voice, music, fileh, static_cast<const tf::bf16*>(w_vhead), static_cast<const tf::bf16*>(b_vhead),
      static_cast<const tf::bf16*>(w_mhead), static_cast<const tf::bf16*>(b_mhead),
      static_cast<const tf::bf16*>(w_file2), static_cast<const tf::bf16*>(b_file2), logits, batch);
  return tf::launch_status();
}

}  // extern "C"

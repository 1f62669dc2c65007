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

}  // extern "C"

// Valid-row transfers between padded device tensors and a packed ("ragged") buffer.
//
// A batch of clips of different lengths is padded to T steps; rows at or past a
// clip's length are never read by the recurrence (its loads stop at the length)
// and its output there is zero. A caller that feeds the GPU from host memory
// therefore only has to move the valid rows across the host link. The packed
// buffer holds, tensor after tensor, each tensor's valid steps:
//
//   tensor i: [B][G_i][T_i][E_i bytes] in device memory (contiguous),
//   packed:   for b in 0..B-1, for g in 0..G_i-1: steps 0..len_b-1 (len_b clamped to
//             [0, T_i]), E_i bytes each; the tensor's region starts at a 16-byte-
//             aligned offset (regions in tensor order, the first at offset 0).
//
// [B, T, ...] tensors (q, k, v, z, angles, out) have G = 1 and E = the row bytes;
// [B, H, T] tensors (adt, dt, trap) have G = H and E = the element size.
// The copy moves raw bytes in either direction (bit-exact), with 16-byte
// vectors where both sides and the length allow it, else 4-byte words, else bytes.
#include <cstdint>

#include "../../include/trifusion_b200.h"
#include "tf_common.cuh"
#include "tf_host.cuh"

namespace tf {
namespace {

constexpr int kMaxTensors = 16;
constexpr int kCopyThreads = 256;

struct RaggedArgs {
  unsigned char* dense[kMaxTensors];
  int64_t groups[kMaxTensors], steps[kMaxTensors], step_bytes[kMaxTensors];
  int ntensors;
};

__device__ __forceinline__ int64_t clamp_len(int64_t len, int64_t t) { return len < 0 ? 0 : (len > t ? t : len); }

__device__ __forceinline__ void copy_bytes(unsigned char* dst, const unsigned char* src, int64_t n) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | static_cast<uintptr_t>(n);
  if ((a & 15) == 0) {
    for (int64_t i = threadIdx.x; i < n / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else if ((a & 3) == 0) {
    for (int64_t i = threadIdx.x; i < n / 4; i += blockDim.x)
      reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
  } else {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}

// CTAs (clip b, slice s of `slices`) x tensor i: slice s of each of clip b's G segments
// (16-byte-aligned slice bounds), so long clips spread over many SMs. Every CTA derives
// its packed offsets from the lengths (O(B) per CTA; B is a batch of clips).
__global__ void __launch_bounds__(kCopyThreads) ragged_copy_kernel(const __grid_constant__ RaggedArgs a,
                                                                   unsigned char* packed, const int64_t* lengths,
                                                                   int batch, int slices, int to_dense) {
  const int i = blockIdx.y, b = blockIdx.x / slices, s = blockIdx.x % slices;
  int64_t base = 0;  // this tensor's region
  for (int j = 0; j < i; ++j) {
    int64_t rows = 0;
    for (int c = 0; c < batch; ++c) rows += clamp_len(lengths[c], a.steps[j]);
    base += (rows * a.groups[j] * a.step_bytes[j] + 15) / 16 * 16;
  }
  const int64_t T = a.steps[i], G = a.groups[i], E = a.step_bytes[i];
  int64_t before = 0;  // valid steps of the clips before b
  for (int c = 0; c < b; ++c) before += clamp_len(lengths[c], T);
  const int64_t len = clamp_len(lengths[b], T);
  if (len == 0) return;
  const int64_t n = len * E;
  const int64_t lo = n * s / slices / 16 * 16, hi = s + 1 == slices ? n : n * (s + 1) / slices / 16 * 16;
  if (hi <= lo) return;
  for (int64_t g = 0; g < G; ++g) {
    unsigned char* p = packed + base + (before * G + g * len) * E + lo;
    unsigned char* d = a.dense[i] + ((static_cast<int64_t>(b) * G + g) * T) * E + lo;
    if (to_dense)
      copy_bytes(d, p, hi - lo);
    else
      copy_bytes(p, d, hi - lo);
  }
}

}  // namespace
}  // namespace tf

extern "C" int tf_ragged_copy_fwd(void* packed, void* const* dense, const int64_t* groups, const int64_t* steps,
                                  const int64_t* step_bytes, int ntensors, const int64_t* lengths, int batch,
                                  int to_dense, void* stream) {
  if (ntensors < 0 || ntensors > tf::kMaxTensors || batch < 0) return TF_ERR_ARG;
  if (ntensors == 0 || batch == 0) return TF_OK;
  if (!packed || !dense || !groups || !steps || !step_bytes || !lengths) return TF_ERR_ARG;
  if (batch > 65535) return TF_ERR_SIZE;
  tf::RaggedArgs a{};
  a.ntensors = ntensors;
  for (int i = 0; i < ntensors; ++i) {
    if (!dense[i] || groups[i] < 0 || steps[i] < 0 || step_bytes[i] < 0) return TF_ERR_ARG;
    a.dense[i] = static_cast<unsigned char*>(dense[i]);
    a.groups[i] = groups[i];
    a.steps[i] = steps[i];
    a.step_bytes[i] = step_bytes[i];
  }
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  // Slices per clip: about two CTAs per SM over the launch (each tensor's segments of a
  // clip split into that many 16-byte-aligned pieces).
  const int64_t want = (2 * static_cast<int64_t>(tf::sm_count()) + batch * ntensors - 1) / (batch * ntensors);
  const int slices = static_cast<int>(want < 1 ? 1 : (want > 256 ? 256 : want));
  if (static_cast<int64_t>(batch) * slices > 2147483647LL) return TF_ERR_SIZE;
  tf::ragged_copy_kernel<<<dim3(batch * slices, ntensors), tf::kCopyThreads, 0,
                           static_cast<cudaStream_t>(stream)>>>(a, static_cast<unsigned char*>(packed), lengths,
                                                                batch, slices, to_dense ? 1 : 0);
  return tf::launch_status();
}

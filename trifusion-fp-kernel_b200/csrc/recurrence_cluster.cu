// Fused Mamba-3 SISO recurrence on the sm_100 tensor cores, chunk-parallel.
//
// Decomposition. Every 64-step chunk of a (batch, head) row is one CTA; the
// CTAs of a row form a thread-block cluster (up to 8 chunks, T <= 512). Each
// chunk works in its own rotary frame: phases accumulate from the chunk start,
// so rotation, scores and the chunk's state contribution
//   dS_c^T = kr_c^T (v_c * scale * 2^(total_c - cs))          (n x p)
// need nothing from earlier chunks. Because q and k of a pair rotate by the
// same angle, the state carried into chunk c, expressed in chunk c's frame, is
//   S(0) = 0,   S(x+1) = R(-theta_x) (2^total_x S(x) + dS_x),
// where theta_x is chunk x's summed angle increment and R rotates the first 32
// (even, odd) pairs of the n axis. Each CTA publishes dS_x, theta_x and
// 2^total_x in its shared memory; after a cluster barrier, chunk c folds its
// predecessors' contributions through distributed shared memory and adds
// (qr_c S(c)^T) 2^cs to its intra-chunk output. In real arithmetic this equals
// the reference's serial recurrence (mamba_fused.py:93-152).
//
// Tensor-core work (tcgen05.mma kind::f16: FP16 operands in 128B-swizzled
// shared memory, FP32 accumulators in tensor memory):
//   scores  D_s  = q16 k16^T              M=64  N=64 K=128
//   state   D_d  = k16^T (vs_hi + vs_lo)  M=128 N=64 K=64 x2  (k16 read MN-major)
//   values  D_pv = (P_hi + P_lo) v16      M=64  N=64 K=64 x2
//   inter   D_i  = q16 S^T                M=64  N=64 K=128
// Precision: FP16 operands carry per-row power-of-two exponents (undone exactly
// after the MMA); the decayed scores P and the decay-weighted values vs are
// split into FP16 hi + lo halves; all sums accumulate in FP32. qk (the D-skip
// dot product, mamba_fused.py:124) is the score diagonal, since rotating q and
// k by the same angle preserves their dot product; the skip term (D + qk) v
// rides on P's diagonal.
#include "recurrence.cuh"
#include "sm100.cuh"

namespace tf {
namespace {

using namespace sm100;

constexpr int kThreads = 256;
constexpr int kMaxCluster = 8;

// Shared-memory map (bytes from a 1024-aligned base).
constexpr uint32_t kOffQ = 0;         // q16  K-major  [2 K-blocks][64 rows][128 B]
constexpr uint32_t kOffK = 16384;     // k16  K-major  [2 K-blocks][64 rows][128 B]; later dS^T export
constexpr uint32_t kOffV = 32768;     // v16  MN-major [64 rows][128 B]
constexpr uint32_t kOffVH = 40960;    // vs hi MN-major; later the z / out tile (BF16 [64][64])
constexpr uint32_t kOffVL = 49152;    // vs lo MN-major
constexpr uint32_t kOffPH = 57344;    // P hi K-major [64 rows][128 B]
constexpr uint32_t kOffPL = 65536;    // P lo
constexpr uint32_t kOffS = 73728;     // S^T MN-major [128 rows][128 B]; prologue: phases FP32 [64][33]
constexpr uint32_t kOffSmall = 90112;

struct Small {
  float cs[kChunk];      // decay cumsum (log2 units)
  float gamma[kChunk];
  float scale[kChunk];
  float dtc[kChunk];
  float qe[kChunk];      // q16 row exponents
  float ke[kChunk];      // k16 row exponents
  float kcoef[kChunk];   // scale_j * 2^-ke_j (score column factor)
  float pe[kChunk];      // P row exponents
  float pmax[2][kChunk];
  float aggexp[2][128];  // 2^-(exponent) of each exported dS^T half-row (read by later chunks)
  float theta[kRotary];  // chunk angle sum mod 2pi (read by later chunks)
  float gtot;            // 2^total (read by later chunks)
  float sinv;            // 2^-(state tile exponent)
  float seg[8][kRotary];
  float wsum[2];
  float red[8];
  uint32_t tmem_base;
  uint32_t pad;
  uint64_t mbar[3];
};
constexpr uint32_t kSmemBytes = kOffSmall + sizeof(Small) + 1024;  // + alignment slack

// TMEM columns (one 256-column allocation per CTA).
constexpr uint32_t kColS = 0, kColD = 64, kColPV = 128, kColI = 192, kTmemCols = 256;

constexpr uint32_t kIdScore = idesc_f16_f32(64, 64, false, false);
constexpr uint32_t kIdState = idesc_f16_f32(128, 64, true, true);
constexpr uint32_t kIdPV = idesc_f16_f32(64, 64, false, true);
constexpr uint32_t kIdInter = idesc_f16_f32(64, 64, false, true);

// ---- small helpers --------------------------------------------------------------
template <int kVec>
__device__ __forceinline__ uint4 load16(const bf16* p) {
  if constexpr (kVec == 16) {
    return __ldg(reinterpret_cast<const uint4*>(p));
  } else if constexpr (kVec == 8) {
    const uint2 a = __ldg(reinterpret_cast<const uint2*>(p));
    const uint2 b = __ldg(reinterpret_cast<const uint2*>(p + 4));
    return make_uint4(a.x, a.y, b.x, b.y);
  } else {
    const unsigned short* s = reinterpret_cast<const unsigned short*>(p);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = static_cast<uint32_t>(s[2 * i]) | (static_cast<uint32_t>(s[2 * i + 1]) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
}
template <int kVec>
__device__ __forceinline__ void store16(bf16* p, uint4 v) {
  if constexpr (kVec == 16) {
    *reinterpret_cast<uint4*>(p) = v;
  } else if constexpr (kVec == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(v.x, v.y);
    *reinterpret_cast<uint2*>(p + 4) = make_uint2(v.z, v.w);
  } else {
    unsigned short* s = reinterpret_cast<unsigned short*>(p);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s[2 * i] = static_cast<unsigned short>(w[i] & 0xffffu);
      s[2 * i + 1] = static_cast<unsigned short>(w[i] >> 16);
    }
  }
}
__device__ __forceinline__ void unpack8(uint4 u, float (&f)[8]) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t a) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(a) : "memory");
}
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr) : "memory");
  return v;
}
// 16 TMEM lanes x 32 columns in the m16n8 fragment order: thread t gets lanes
// t/4 and t/4+8, columns 8k + 2(t%4) + {0,1} for k = 0..3, as
// r[4k + 0..1] (lane t/4) and r[4k + 2..3] (lane t/4 + 8).
__device__ __forceinline__ void tmem_ld_16x256_x4(uint32_t taddr, float (&r)[16]) {
  uint32_t* u = reinterpret_cast<uint32_t*>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
        "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void bar_sync_n(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ float load_trap(const RecurrenceParams& p, const char* base, int64_t off) {
  return p.trap_bf16 ? bf2f(reinterpret_cast<const bf16*>(base)[off]) : reinterpret_cast<const float*>(base)[off];
}
// floor(log2 |x|) of the largest magnitude, or a sentinel for zero rows.
__device__ __forceinline__ int ilog2_or(float max_abs, int if_zero) {
  if (!(max_abs > 0.f)) return if_zero;
  return static_cast<int>((__float_as_uint(max_abs) >> 23) & 0xffu) - 127;
}
__device__ __forceinline__ float silu_tanh(float z) {
  const float hz = 0.5f * z;
  return fmaf(hz, tanh_approx(hz), hz);  // z * sigmoid(z) = hz * (1 + tanh(hz))
}

__device__ int g_device_error = 0;  // set when a bounded wait gives up

template <int kVec>
__global__ void __launch_bounds__(kThreads, 2) recurrence_cluster_kernel(RecurrenceParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  unsigned char* smem = smem_raw + (base - raw_addr);
  Small& sm = *reinterpret_cast<Small*>(smem + kOffSmall);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int quarter = warp & 3, chalf = warp >> 2;  // TMEM lane quarter; column half
  const int c = static_cast<int>(cluster_ctarank());
  const int b = blockIdx.y / p.H, h = blockIdx.y % p.H;
  const int qh = h / (p.H / p.Hq);
  int T_eff = p.T;
  if (p.lengths) {
    const int64_t len = p.lengths[b];
    T_eff = static_cast<int>(len < 0 ? 0 : (len > p.T ? p.T : len));
  }
  const int c0 = c * kChunk;
  const int nv = max(0, min(kChunk, T_eff - c0));  // valid rows in this chunk

  if (warp == 0) {
    tmem_alloc(&sm.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) mbar_init(&sm.mbar[i], 1);
    fence_mbar_init();
  }

  // ---- prefetch: row t = tid/4, sub-slot s = tid%4 ---------------------------
  // q/k elements {8s, 32+8s} (rotating pairs 4s..4s+3, 16+4s..16+4s+3) and
  // {64+8s, 96+8s} (phase 0); v and z elements {8s, 32+8s}.
  const int t = tid >> 2, s = tid & 3;
  const bool row_ok = t < nv;
  uint4 qraw[4], kraw[4], vraw[2], zraw[2];
  {
    const int64_t pos = c0 + t;
    const bf16* qrow = p.q + b * p.sq[0] + pos * p.sq[1] + qh * p.sq[2];
    const bf16* krow = p.k + b * p.sk[0] + pos * p.sk[1] + qh * p.sk[2];
    const bf16* vrow = p.v + b * p.sv[0] + pos * p.sv[1] + h * p.sv[2];
    const bf16* zrow = p.z + b * p.sz[0] + pos * p.sz[1] + h * p.sz[2];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = 32 * i + 8 * s;
      qraw[i] = row_ok ? load16<kVec>(qrow + e) : make_uint4(0, 0, 0, 0);
      kraw[i] = row_ok ? load16<kVec>(krow + e) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int e = 32 * i + 8 * s;
      vraw[i] = row_ok ? load16<kVec>(vrow + e) : make_uint4(0, 0, 0, 0);
      zraw[i] = row_ok ? load16<kVec>(zrow + e) : make_uint4(0, 0, 0, 0);
    }
  }

  // Controls (threads 0..63, one step each) and this thread's 8 raw angles
  // (lane = pair r, warp = 8-step segment), loaded up front with q/k/v/z.
  float c_dt = 0.f, c_dn = 0.f, c_tr = 0.f, c_tn = 0.f, c_adt = 0.f;
  if (tid < kChunk) {
    const float* dtbase = p.dt + b * p.sdt[0] + h * p.sdt[1];
    const float* adtbase = p.adt + b * p.sadt[0] + h * p.sadt[1];
    const char* trbase = static_cast<const char*>(p.trap) + (b * p.str[0] + h * p.str[1]) * (p.trap_bf16 ? 2 : 4);
    const int64_t tt = c0 + tid;
    const bool valid = tid < nv;
    const bool next = tt + 1 < T_eff;
    if (valid) {
      c_dt = dtbase[tt * p.sdt[2]];
      c_tr = load_trap(p, trbase, tt * p.str[2]);
      c_adt = adtbase[tt * p.sadt[2]];
    }
    if (next) {
      c_dn = dtbase[(tt + 1) * p.sdt[2]];
      c_tn = load_trap(p, trbase, (tt + 1) * p.str[2]);
    }
  }
  float araw[8];
  {
    const bf16* abase = p.ang + b * p.sa[0] + h * p.sa[2];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int tt = warp * 8 + i;
      araw[i] = tt < nv ? bf2f(abase[static_cast<int64_t>(c0 + tt) * p.sa[1] + lane * p.sa[3]]) : 0.f;
    }
  }
  if (tid < kChunk) {
    const float trv = sigmoidf_fast(c_tr);
    const float tnv = sigmoidf_fast(c_tn);
    const float gm = c_dt * trv;
    float x = c_adt * kLog2e;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) sm.wsum[warp] = x;
    sm.dtc[tid] = c_dt;
    sm.gamma[tid] = gm;
    sm.scale[tid] = c_dn * (1.f - tnv) + gm;
    sm.cs[tid] = x;
  }
  __syncthreads();
  if (tid >= 32 && tid < kChunk) sm.cs[tid] += sm.wsum[0];

  // ---- local angle phases: lane = pair r, warp = 8-step segment ------------
  float* phase = reinterpret_cast<float*>(smem + kOffS);  // [64][33]
  {
    const int r = lane, t0 = warp * 8;
    float run = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int tt = t0 + i;
      run = fmaf(tanh_approx(araw[i]) * kPi, sm.dtc[tt], run);
      phase[tt * 33 + r] = run;
    }
    sm.seg[warp][r] = run;
  }
  __syncthreads();
  {
    const int r = lane, t0 = warp * 8;
    float off = 0.f;
    for (int q = 0; q < warp; ++q) off += sm.seg[q][r];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float ph = phase[(t0 + i) * 33 + r] + off;
      phase[(t0 + i) * 33 + r] = ph - kTwoPi * floorf(ph * (1.f / kTwoPi));
    }
    if (warp == 0) {
      float th = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q) th += sm.seg[q][r];
      sm.theta[r] = th - kTwoPi * floorf(th * (1.f / kTwoPi));
    }
  }
  __syncthreads();
  const float total = sm.cs[kChunk - 1];
  if (tid == 0) sm.gtot = ex2_approx(total);

  // ---- rows -> FP16 operand tiles --------------------------------------------
  {
    const float* qbh = p.qb + h * kState;
    const float* kbh = p.kb + h * kState;
    // q: optional C_norm, bias, rotation, row exponent.
    float x[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[8];
      unpack8(qraw[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[8 * i + e] = f[e];
    }
    if (p.qw) {  // RMSNorm with FP32 statistics, BF16 result (native.py:8-39)
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 32; ++e) ss = fmaf(x[e], x[e], ss);
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      const float rr = rsqrtf(ss * (1.f / kState) + p.eps);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) x[8 * i + e] = bf16_round((x[8 * i + e] * rr) * p.qw[32 * i + 8 * s + e]);
    }
    float cn[8], sn[8];  // this thread's 8 rotating pairs
#pragma unroll
    for (int m = 0; m < 8; ++m) __sincosf(phase[t * 33 + (m < 4 ? 4 * s + m : 16 + 4 * s + m - 4)], &sn[m], &cn[m]);
    float qmax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[8 * i + e] = row_ok ? x[8 * i + e] + qbh[32 * i + 8 * s + e] : 0.f;
      if (i < 2) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float a0 = x[8 * i + 2 * m], a1 = x[8 * i + 2 * m + 1];
          const float cc = cn[4 * i + m], ssn = sn[4 * i + m];
          x[8 * i + 2 * m] = a0 * cc - a1 * ssn;
          x[8 * i + 2 * m + 1] = a0 * ssn + a1 * cc;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) qmax = fmaxf(qmax, fabsf(x[8 * i + e]));
    }
    qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 1));
    qmax = fmaxf(qmax, __shfl_xor_sync(0xffffffffu, qmax, 2));
    const int qe = pow2_scale_exponent(qmax);
    {
      const float qs = exp2i(qe);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int e0 = 32 * i + 8 * s;
        st_shared_v4(base + kOffQ + (e0 >> 6) * 8192u + sw128_offset(t, e0 & 63),
                     pack_f16x2(x[8 * i] * qs, x[8 * i + 1] * qs), pack_f16x2(x[8 * i + 2] * qs, x[8 * i + 3] * qs),
                     pack_f16x2(x[8 * i + 4] * qs, x[8 * i + 5] * qs), pack_f16x2(x[8 * i + 6] * qs, x[8 * i + 7] * qs));
      }
    }
    // k: optional B_norm, bias, rotation.
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float f[8];
      unpack8(kraw[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[8 * i + e] = f[e];
    }
    if (p.kw) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 32; ++e) ss = fmaf(x[e], x[e], ss);
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      const float rr = rsqrtf(ss * (1.f / kState) + p.eps);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int e = 0; e < 8; ++e) x[8 * i + e] = bf16_round((x[8 * i + e] * rr) * p.kw[32 * i + 8 * s + e]);
    }
    float kmax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[8 * i + e] = row_ok ? x[8 * i + e] + kbh[32 * i + 8 * s + e] : 0.f;
      if (i < 2) {
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float a0 = x[8 * i + 2 * m], a1 = x[8 * i + 2 * m + 1];
          const float cc = cn[4 * i + m], ssn = sn[4 * i + m];
          x[8 * i + 2 * m] = a0 * cc - a1 * ssn;
          x[8 * i + 2 * m + 1] = a0 * ssn + a1 * cc;
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) kmax = fmaxf(kmax, fabsf(x[8 * i + e]));
    }
    kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, 1));
    kmax = fmaxf(kmax, __shfl_xor_sync(0xffffffffu, kmax, 2));
    // v and the decay-weighted v of the state update.
    float vf[16];
    unpack8(vraw[0], *reinterpret_cast<float(*)[8]>(&vf[0]));
    unpack8(vraw[1], *reinterpret_cast<float(*)[8]>(&vf[8]));
    float vmax = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) vmax = fmaxf(vmax, fabsf(vf[e]));
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
    vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
    const float sw = row_ok ? sm.scale[t] * ex2_approx(total - sm.cs[t]) : 0.f;
    // Split 2^a between k16 = kr 2^a and vs = v scale w 2^-a so both sit near
    // the geometric mean of their magnitudes, inside FP16's normal range.
    const int kl = ilog2_or(kmax, 1000), vl = ilog2_or(vmax * sw, 1000);
    int ka = 0;
    if (kl != 1000) ka = vl != 1000 ? ((vl - kl) >> 1) : 14 - kl;
    ka = ka < -60 ? -60 : (ka > 60 ? 60 : ka);
    {
      const float ks = exp2i(ka);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int e0 = 32 * i + 8 * s;
        st_shared_v4(base + kOffK + (e0 >> 6) * 8192u + sw128_offset(t, e0 & 63),
                     pack_f16x2(x[8 * i] * ks, x[8 * i + 1] * ks), pack_f16x2(x[8 * i + 2] * ks, x[8 * i + 3] * ks),
                     pack_f16x2(x[8 * i + 4] * ks, x[8 * i + 5] * ks), pack_f16x2(x[8 * i + 6] * ks, x[8 * i + 7] * ks));
      }
      const float vsc = sw * exp2i(-ka);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const uint32_t off = sw128_offset(t, 32 * i + 8 * s);
        uint32_t hv[4], hh[4], hl[4];
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float a0 = vf[8 * i + 2 * m], a1 = vf[8 * i + 2 * m + 1];
          hv[m] = pack_f16x2(a0, a1);
          const float w0 = a0 * vsc, w1 = a1 * vsc;
          hh[m] = pack_f16x2(w0, w1);
          const float2 back = unpack_f16x2(hh[m]);
          hl[m] = pack_f16x2(w0 - back.x, w1 - back.y);
        }
        st_shared_v4(base + kOffV + off, hv[0], hv[1], hv[2], hv[3]);
        st_shared_v4(base + kOffVH + off, hh[0], hh[1], hh[2], hh[3]);
        st_shared_v4(base + kOffVL + off, hl[0], hl[1], hl[2], hl[3]);
      }
    }
    if (s == 0) {
      sm.qe[t] = static_cast<float>(qe);
      sm.ke[t] = static_cast<float>(ka);
      sm.kcoef[t] = sm.scale[t] * exp2i(-ka);
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // ---- MMA 1: scores and the chunk's state contribution --------------------
  if (tid == 0) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t koff = (kk >> 2) * 8192u + (kk & 3) * 32u;
      umma_f16(tmem + kColS, desc_sw128(base + kOffQ + koff, 0, 1024), desc_sw128(base + kOffK + koff, 0, 1024),
               kIdScore, kk > 0);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      umma_f16(tmem + kColD, desc_sw128(base + kOffK + kk * 2048u, 8192, 1024),
               desc_sw128(base + kOffVH + kk * 2048u, 8192, 1024), kIdState, kk > 0);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      umma_f16(tmem + kColD, desc_sw128(base + kOffK + kk * 2048u, 8192, 1024),
               desc_sw128(base + kOffVL + kk * 2048u, 8192, 1024), kIdState, 1);
    }
    umma_commit(&sm.mbar[0]);
  }
  bool ok = mbar_wait(&sm.mbar[0], 0);
  tc_fence_after();

  // z tile (BF16 [64][64], 16-byte chunks swizzled by row) over the dead vs-hi tile.
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t off = sw128_offset(t, 32 * i + 8 * s);
    st_shared_v4(base + kOffVH + off, zraw[i].x, zraw[i].y, zraw[i].z, zraw[i].w);
  }

  // ---- export dS^T (row n, 32-column half) as FP16 with a per-half-row exponent
  {
    const uint32_t n = 32 * quarter + lane;
    float r[32];
    tmem_ld16(tmem_addr(tmem, 32 * quarter, kColD + 32 * chalf), *reinterpret_cast<float(*)[16]>(&r[0]));
    tmem_ld16(tmem_addr(tmem, 32 * quarter, kColD + 32 * chalf + 16), *reinterpret_cast<float(*)[16]>(&r[16]));
    tmem_wait_ld();
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) m = fmaxf(m, fabsf(r[j]));
    const int ae = pow2_scale_exponent(m);
    const float as = exp2i(ae);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t ch = (4u * chalf + k) ^ (n & 7u);
      st_shared_v4(base + kOffK + n * 128u + ch * 16u, pack_f16x2(r[8 * k] * as, r[8 * k + 1] * as),
                   pack_f16x2(r[8 * k + 2] * as, r[8 * k + 3] * as), pack_f16x2(r[8 * k + 4] * as, r[8 * k + 5] * as),
                   pack_f16x2(r[8 * k + 6] * as, r[8 * k + 7] * as));
    }
    sm.aggexp[chalf][n] = exp2i(-ae);
  }

  // ---- decayed scores P (+ the D-skip diagonal) -> FP16 hi/lo tiles ----------
  const int g = lane >> 2, c4 = lane & 3;
  const int i0 = 16 * quarter + g, i1 = i0 + 8;
  {
    float sc[16];
    tmem_ld_16x256_x4(tmem_addr(tmem, 32 * quarter, kColS + 32 * chalf), sc);
    tmem_wait_ld();
    const float d = p.d[h];
    const float cs0 = sm.cs[i0], cs1 = sm.cs[i1];
    const float rq0 = cs0 - sm.qe[i0], rq1 = cs1 - sm.qe[i1];
    const float dg0 = exp2i(-static_cast<int>(sm.qe[i0]) - static_cast<int>(sm.ke[i0])) * sm.gamma[i0];
    const float dg1 = exp2i(-static_cast<int>(sm.qe[i1]) - static_cast<int>(sm.ke[i1])) * sm.gamma[i1];
    float m0 = 0.f, m1 = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 32 * chalf + 8 * k + 2 * c4 + e;
        const float kc = sm.kcoef[j], csj = sm.cs[j];
        float v0 = sc[4 * k + e], v1 = sc[4 * k + 2 + e];
        v0 = j < i0 ? v0 * kc * ex2_approx(rq0 - csj) : (j == i0 ? d + v0 * dg0 : 0.f);
        v1 = j < i1 ? v1 * kc * ex2_approx(rq1 - csj) : (j == i1 ? d + v1 * dg1 : 0.f);
        sc[4 * k + e] = v0;
        sc[4 * k + 2 + e] = v1;
        m0 = fmaxf(m0, fabsf(v0));
        m1 = fmaxf(m1, fabsf(v1));
      }
    }
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
    m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
    m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
    if (c4 == 0) {
      sm.pmax[chalf][i0] = m0;
      sm.pmax[chalf][i1] = m1;
    }
    bar_sync_n(1 + quarter, 64);  // the two warps sharing this TMEM quarter
    m0 = fmaxf(sm.pmax[0][i0], sm.pmax[1][i0]);
    m1 = fmaxf(sm.pmax[0][i1], sm.pmax[1][i1]);
    const int pe0 = pow2_scale_exponent(m0), pe1 = pow2_scale_exponent(m1);
    if (chalf == 0 && c4 == 0) {
      sm.pe[i0] = static_cast<float>(pe0);
      sm.pe[i1] = static_cast<float>(pe1);
    }
    const float ps0 = exp2i(pe0), ps1 = exp2i(pe1);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 32 * chalf + 8 * k + 2 * c4;
      const float a0 = sc[4 * k] * ps0, a1 = sc[4 * k + 1] * ps0;
      const float b0 = sc[4 * k + 2] * ps1, b1 = sc[4 * k + 3] * ps1;
      const uint32_t h0 = pack_f16x2(a0, a1), h1 = pack_f16x2(b0, b1);
      const float2 f0 = unpack_f16x2(h0), f1 = unpack_f16x2(h1);
      st_shared_u32(base + kOffPH + sw128_offset(i0, j), h0);
      st_shared_u32(base + kOffPH + sw128_offset(i1, j), h1);
      st_shared_u32(base + kOffPL + sw128_offset(i0, j), pack_f16x2(a0 - f0.x, a1 - f0.y));
      st_shared_u32(base + kOffPL + sw128_offset(i1, j), pack_f16x2(b0 - f1.x, b1 - f1.y));
    }
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // ---- MMA 2: values ---------------------------------------------------------------
  if (tid == 0) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      umma_f16(tmem + kColPV, desc_sw128(base + kOffPH + kk * 32u, 0, 1024),
               desc_sw128(base + kOffV + kk * 2048u, 8192, 1024), kIdPV, kk > 0);
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      umma_f16(tmem + kColPV, desc_sw128(base + kOffPL + kk * 32u, 0, 1024),
               desc_sw128(base + kOffV + kk * 2048u, 8192, 1024), kIdPV, 1);
    }
    umma_commit(&sm.mbar[1]);
  }

  // ---- publish, then fold the predecessors' state contributions --------------
  cluster_sync();
  if (c > 0) {
    const uint32_t n = 32 * quarter + lane;
    float st[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) st[j] = 0.f;
    const uint32_t agg_row = base + kOffK + n * 128u;
    const uint32_t small_local = base + kOffSmall;
    // Remote loads of predecessor x are all issued before any of them is used.
    uint4 u[4];
    float gx, fx, th;
    auto fetch = [&](int x) {
      const uint32_t rs = map_shared(small_local, x);
      const uint32_t ra = map_shared(agg_row, x);
#pragma unroll
      for (int k = 0; k < 4; ++k) u[k] = ld_dsmem_v4(ra + (((4u * chalf + k) ^ (n & 7u)) << 4));
      gx = ld_dsmem_f32(rs + offsetof(Small, gtot));
      fx = ld_dsmem_f32(rs + offsetof(Small, aggexp) + 4u * (128u * chalf + n));
      th = ld_dsmem_f32(rs + offsetof(Small, theta) + 4u * ((n >> 1) & 31u));
    };
    fetch(0);
    for (int x = 0; x < c; ++x) {
      float val[32];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t w[4] = {u[k].x, u[k].y, u[k].z, u[k].w};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const float2 f = unpack_f16x2(w[m]);
          val[8 * k + 2 * m] = f.x;
          val[8 * k + 2 * m + 1] = f.y;
        }
      }
      const float g_x = gx, f_x = fx, th_x = th;
      if (x + 1 < c) fetch(x + 1);
#pragma unroll
      for (int j = 0; j < 32; ++j) st[j] = fmaf(g_x, st[j], val[j] * f_x);
      if (quarter < 2) {  // rows n < 64 hold the 32 rotating pairs (2r, 2r+1)
        float snx, cnx;
        __sincosf(th_x, &snx, &cnx);
        const float sgn = (n & 1u) ? -snx : snx;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float other = __shfl_xor_sync(0xffffffffu, st[j], 1);
          // R(-theta): (a, b) -> (a cos + b sin, b cos - a sin)
          st[j] = fmaf(st[j], cnx, other * sgn);
        }
      }
    }
    float m = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) m = fmaxf(m, fabsf(st[j]));
    m = warp_max(m);
    if (lane == 0) sm.red[warp] = m;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < 8; ++w) m = fmaxf(m, sm.red[w]);
    const int se = pow2_scale_exponent(m);
    const float ss = exp2i(se);
    if (tid == 0) sm.sinv = exp2i(-se);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      st_shared_v4(base + kOffS + sw128_offset(n, 32 * chalf + 8 * k), pack_f16x2(st[8 * k] * ss, st[8 * k + 1] * ss),
                   pack_f16x2(st[8 * k + 2] * ss, st[8 * k + 3] * ss), pack_f16x2(st[8 * k + 4] * ss, st[8 * k + 5] * ss),
                   pack_f16x2(st[8 * k + 6] * ss, st[8 * k + 7] * ss));
    }
  }
  cluster_sync();  // every chunk is done reading its predecessors' shared memory
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // ---- MMA 3: inter-chunk term -------------------------------------------------
  if (tid == 0 && c > 0) {
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t koff = (kk >> 2) * 8192u + (kk & 3) * 32u;
      umma_f16(tmem + kColI, desc_sw128(base + kOffQ + koff, 0, 1024),
               desc_sw128(base + kOffS + kk * 2048u, 8192, 1024), kIdInter, kk > 0);
    }
    umma_commit(&sm.mbar[2]);
  }

  // ---- output: combine, gate, stage in the z tile ------------------------------
  ok &= mbar_wait(&sm.mbar[1], 0);
  if (c > 0) ok &= mbar_wait(&sm.mbar[2], 0);
  tc_fence_after();
  {
    float pv[16], it[16];
    tmem_ld_16x256_x4(tmem_addr(tmem, 32 * quarter, kColPV + 32 * chalf), pv);
    if (c > 0) tmem_ld_16x256_x4(tmem_addr(tmem, 32 * quarter, kColI + 32 * chalf), it);
    tmem_wait_ld();
    const float u0 = exp2i(-static_cast<int>(sm.pe[i0])), u1 = exp2i(-static_cast<int>(sm.pe[i1]));
    const float w0 = c > 0 ? ex2_approx(sm.cs[i0] - sm.qe[i0]) * sm.sinv : 0.f;
    const float w1 = c > 0 ? ex2_approx(sm.cs[i1] - sm.qe[i1]) * sm.sinv : 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 32 * chalf + 8 * k + 2 * c4;
      const uint32_t a0 = base + kOffVH + sw128_offset(i0, j), a1 = base + kOffVH + sw128_offset(i1, j);
      const float2 z0 = unpack_bf16x2(ld_shared_u32(a0)), z1 = unpack_bf16x2(ld_shared_u32(a1));
      float o[4];
      o[0] = pv[4 * k] * u0 + (c > 0 ? it[4 * k] * w0 : 0.f);
      o[1] = pv[4 * k + 1] * u0 + (c > 0 ? it[4 * k + 1] * w0 : 0.f);
      o[2] = pv[4 * k + 2] * u1 + (c > 0 ? it[4 * k + 2] * w1 : 0.f);
      o[3] = pv[4 * k + 3] * u1 + (c > 0 ? it[4 * k + 3] * w1 : 0.f);
      st_shared_u32(a0, pack_bf16x2(o[0] * silu_tanh(z0.x), o[1] * silu_tanh(z0.y)));
      st_shared_u32(a1, pack_bf16x2(o[2] * silu_tanh(z1.x), o[3] * silu_tanh(z1.y)));
    }
  }
  __syncthreads();
  // Coalesced row stores; rows past the length are zero (their z, v are zero).
  if (c0 + t < p.T) {
    bf16* orow = p.out + b * p.so[0] + static_cast<int64_t>(c0 + t) * p.so[1] + h * p.so[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int e = 32 * i + 8 * s;
      const uint4 val = row_ok ? ld_shared_v4(base + kOffVH + sw128_offset(t, e)) : make_uint4(0, 0, 0, 0);
      store16<kVec>(orow + e, val);
    }
  }
  if (!ok) atomicExch(&g_device_error, 1);

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

int alignment_class(const RecurrenceParams& p) {
  auto rows_aligned = [](const void* ptr, const int64_t* st, int nd, int bytes) {
    if (reinterpret_cast<uintptr_t>(ptr) % bytes) return false;
    for (int i = 0; i < nd; ++i)
      if ((st[i] * 2) % bytes) return false;
    return true;
  };
  for (int bytes : {16, 8}) {
    if (rows_aligned(p.q, p.sq, 3, bytes) && rows_aligned(p.k, p.sk, 3, bytes) &&
        rows_aligned(p.v, p.sv, 3, bytes) && rows_aligned(p.z, p.sz, 3, bytes) &&
        rows_aligned(p.out, p.so, 3, bytes))
      return bytes;
  }
  return 2;
}

template <int kVec>
int launch_cluster(const RecurrenceParams& p, int nck, cudaStream_t stream) {
  auto kernel = recurrence_cluster_kernel<kVec>;
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nck, p.B * p.H, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = nck;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, p) == cudaSuccess ? 0 : -1;
}

}  // namespace

bool cluster_path_supported(const RecurrenceParams& p) {
  const int nck = (p.T + kChunk - 1) / kChunk;
  return nck >= 1 && nck <= kMaxCluster;
}

int launch_recurrence_cluster(const RecurrenceParams& p, cudaStream_t stream) {
  const int nck = (p.T + kChunk - 1) / kChunk;
  switch (alignment_class(p)) {
    case 16: return launch_cluster<16>(p, nck, stream);
    case 8: return launch_cluster<8>(p, nck, stream);
    default: return launch_cluster<2>(p, nck, stream);
  }
}

int read_device_error(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
  }
  return v;
}

}  // namespace tf

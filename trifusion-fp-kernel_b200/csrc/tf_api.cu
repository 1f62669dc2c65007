// C ABI of trifusion_b200: argument validation, status codes and launches.
// Declarations and the reference interface each entry point replaces are in
// include/trifusion_b200.h.
#include <atomic>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/trifusion_b200.h"
#include "recurrence.cuh"
#include "tf_host.cuh"

namespace tf {

thread_local char g_last_error[256] = "";

// Per-device "is sm_100" cache: 0 = unknown, 1 = yes, 2 = no. Filled on the
// first call for a device; later calls only read it (safe under graph capture).
constexpr int kMaxDevices = 64;
int g_arch_ok[kMaxDevices] = {0};

int check_device() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    snprintf(g_last_error, sizeof g_last_error, "%s", cudaGetErrorString(e));
    return TF_ERR_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return TF_ERR_DEVICE;
  if (g_arch_ok[dev] == 0) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    g_arch_ok[dev] = (major == 10 && minor == 0) ? 1 : 2;
  }
  return g_arch_ok[dev] == 1 ? TF_OK : TF_ERR_DEVICE;
}

int g_sm_count[kMaxDevices] = {0};

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  }
  return g_sm_count[dev];
}

// Host-mapped error word (pinned, written by kernels whose bounded wait gave up)
// and the flag-wait limit of later launches.
std::atomic<int*> g_host_error{nullptr};
std::atomic<unsigned long long> g_flag_wait_ns{2000000000ull};

int* host_error_word() { return g_host_error.load(std::memory_order_relaxed); }
unsigned long long flag_wait_limit_ns() { return g_flag_wait_ns.load(std::memory_order_relaxed); }

int launch_status() {
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return TF_OK;
  snprintf(g_last_error, sizeof g_last_error, "%s", cudaGetErrorString(e));
  return TF_ERR_LAUNCH;
}

// Builds and validates the parameters of a one-direction launch. Returns TF_OK
// (with `empty` set when there is nothing to launch) or an error status; touches
// no device state besides the per-device attribute cache.
int recurrence_params(const void* q, const void* k, const void* v, const float* adt, const float* dt,
                      const void* trap, int trap_dtype, const float* qb, const float* kb, const void* angles,
                      const float* d, const void* z, void* out, const int64_t* strides, int batch, int seqlen,
                      int heads, int groups, const float* qw, const float* kw, float eps,
                      const int64_t* lengths, RecurrenceParams& p, bool& empty) {
  empty = false;
  if (!strides || batch < 0 || seqlen < 0 || heads < 0 || groups <= 0) return TF_ERR_ARG;
  if (trap_dtype != TF_F32 && trap_dtype != TF_BF16) return TF_ERR_ARG;
  if (heads % groups != 0) return TF_ERR_ARG;
  if (batch == 0 || seqlen == 0 || heads == 0) {  // empty launch grid
    empty = true;
    return TF_OK;
  }
  if (!q || !k || !v || !adt || !dt || !trap || !qb || !kb || !angles || !d || !z || !out)
    return TF_ERR_ARG;
  p = RecurrenceParams{};
  p.q = static_cast<const bf16*>(q);
  p.k = static_cast<const bf16*>(k);
  p.v = static_cast<const bf16*>(v);
  p.z = static_cast<const bf16*>(z);
  p.ang = static_cast<const bf16*>(angles);
  p.adt = adt;
  p.dt = dt;
  p.trap = trap;
  p.trap_bf16 = trap_dtype == TF_BF16;
  p.qb = qb;
  p.kb = kb;
  p.d = d;
  p.qw = qw;
  p.kw = kw;
  p.eps = eps;
  p.lengths = lengths;
  p.out = static_cast<bf16*>(out);
  const int64_t* s = strides;
  for (int i = 0; i < 4; ++i) p.sq[i] = s[i];
  for (int i = 0; i < 4; ++i) p.sk[i] = s[4 + i];
  for (int i = 0; i < 4; ++i) p.sv[i] = s[8 + i];
  for (int i = 0; i < 3; ++i) p.sadt[i] = s[12 + i];
  for (int i = 0; i < 3; ++i) p.sdt[i] = s[15 + i];
  for (int i = 0; i < 3; ++i) p.str[i] = s[18 + i];
  for (int i = 0; i < 4; ++i) p.sa[i] = s[21 + i];
  for (int i = 0; i < 4; ++i) p.sz[i] = s[25 + i];
  for (int i = 0; i < 4; ++i) p.so[i] = s[29 + i];
  // The innermost dimension of q, k, v, z and out must be contiguous.
  if (p.sq[3] != 1 || p.sk[3] != 1 || p.sv[3] != 1 || p.sz[3] != 1 || p.so[3] != 1)
    return TF_ERR_LAYOUT;
  p.B = batch;
  p.T = seqlen;
  p.H = heads;
  p.Hq = groups;
  return check_device();
}

// Launches validated one-direction parameters on `workspace`.
int recurrence_launch(const RecurrenceParams& p, void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace) return TF_ERR_ARG;
  if (workspace_bytes < recurrence_workspace_bytes(p.B, p.T, p.H)) return TF_ERR_SIZE;
  RecurrenceLaunch launch{};
  launch.dir[0] = p;
  launch.dir[1] = p;
  launch.ndir = 1;
  const int st = launch_recurrence_persistent(launch, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
  if (st != 0) {
    const int ls = launch_status();
    return ls != TF_OK ? ls : TF_ERR_LAUNCH;
  }
  return launch_status();
}

int recurrence_entry(const void* q, const void* k, const void* v, const float* adt,
                     const float* dt, const void* trap, int trap_dtype, const float* qb,
                     const float* kb, const void* angles, const float* d, const void* z,
                     void* out, const int64_t* strides, int batch, int seqlen, int heads,
                     int groups, const float* qw, const float* kw, float eps,
                     const int64_t* lengths, void* workspace, size_t workspace_bytes, void* stream) {
  RecurrenceParams p;
  bool empty = false;
  const int st = recurrence_params(q, k, v, adt, dt, trap, trap_dtype, qb, kb, angles, d, z, out, strides, batch,
                                   seqlen, heads, groups, qw, kw, eps, lengths, p, empty);
  if (st != TF_OK || empty) return st;
  return recurrence_launch(p, workspace, workspace_bytes, stream);
}

// One direction's parameters from the public argument record; validation as in
// recurrence_entry. Returns TF_OK or an error status.
int params_from_io(const tf_recurrence_io& io, int batch, int seqlen, int heads, int groups, float eps,
                   const int64_t* lengths, RecurrenceParams& p) {
  if (io.trap_dtype != TF_F32 && io.trap_dtype != TF_BF16) return TF_ERR_ARG;
  const bool raw = io.a_raw != nullptr || io.ddt_raw != nullptr;
  if (raw && (!io.a_raw || !io.ddt_raw || !io.dt_bias)) return TF_ERR_ARG;
  if (!raw && (!io.adt || !io.dt)) return TF_ERR_ARG;
  if (!io.q || !io.k || !io.v || !io.z || !io.angles || !io.trap || !io.qb || !io.kb || !io.d || !io.out)
    return TF_ERR_ARG;
  p = RecurrenceParams{};
  p.q = static_cast<const bf16*>(io.q);
  p.k = static_cast<const bf16*>(io.k);
  p.v = static_cast<const bf16*>(io.v);
  p.z = static_cast<const bf16*>(io.z);
  p.ang = static_cast<const bf16*>(io.angles);
  p.adt = io.adt;
  p.dt = io.dt;
  p.trap = io.trap;
  p.trap_bf16 = io.trap_dtype == TF_BF16;
  p.qb = io.qb;
  p.kb = io.kb;
  p.d = io.d;
  p.qw = io.q_norm_w;
  p.kw = io.k_norm_w;
  p.eps = eps;
  p.lengths = lengths;
  p.out = static_cast<bf16*>(io.out);
  const int64_t* s = io.strides;
  for (int i = 0; i < 4; ++i) p.sq[i] = s[i];
  for (int i = 0; i < 4; ++i) p.sk[i] = s[4 + i];
  for (int i = 0; i < 4; ++i) p.sv[i] = s[8 + i];
  for (int i = 0; i < 3; ++i) p.sadt[i] = s[12 + i];
  for (int i = 0; i < 3; ++i) p.sdt[i] = s[15 + i];
  for (int i = 0; i < 3; ++i) p.str[i] = s[18 + i];
  for (int i = 0; i < 4; ++i) p.sa[i] = s[21 + i];
  for (int i = 0; i < 4; ++i) p.sz[i] = s[25 + i];
  for (int i = 0; i < 4; ++i) p.so[i] = s[29 + i];
  for (int i = 0; i < 3; ++i) p.sar[i] = s[33 + i];
  for (int i = 0; i < 3; ++i) p.sdr[i] = s[36 + i];
  if (p.sq[3] != 1 || p.sk[3] != 1 || p.sv[3] != 1 || p.sz[3] != 1 || p.so[3] != 1) return TF_ERR_LAYOUT;
  p.raw_controls = raw ? 1 : 0;
  p.a_raw = static_cast<const bf16*>(io.a_raw);
  p.ddt_raw = static_cast<const bf16*>(io.ddt_raw);
  p.dt_bias = io.dt_bias;
  p.a_floor = io.a_floor;
  p.reverse = io.reverse ? 1 : 0;
  p.B = batch;
  p.T = seqlen;
  p.H = heads;
  p.Hq = groups;
  return TF_OK;
}

}  // namespace tf

extern "C" {

size_t tf_recurrence_workspace_size_multi(int count, int batch, int seqlen, int heads) {
  if (count < 1 || count > 2 || batch <= 0 || seqlen <= 0 || heads <= 0) return 0;
  return tf::recurrence_workspace_bytes(batch, seqlen, heads, count);
}

int tf_mamba_recurrence_multi_fwd(const tf_recurrence_io* io, int count, int batch, int seqlen,
                                  int heads, int groups, float eps, const int64_t* lengths,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (!io || count < 1 || count > 2) return TF_ERR_ARG;
  if (batch < 0 || seqlen < 0 || heads < 0 || groups <= 0 || heads % groups) return TF_ERR_ARG;
  if (batch == 0 || seqlen == 0 || heads == 0) return TF_OK;
  tf::RecurrenceLaunch launch{};
  for (int i = 0; i < count; ++i) {
    const int st = tf::params_from_io(io[i], batch, seqlen, heads, groups, eps, lengths, launch.dir[i]);
    if (st != TF_OK) return st;
  }
  if (count == 1) launch.dir[1] = launch.dir[0];
  launch.ndir = count;
  const int st = tf::check_device();
  if (st != TF_OK) return st;
  if (!workspace) return TF_ERR_ARG;
  if (workspace_bytes < tf::recurrence_workspace_bytes(batch, seqlen, heads, count)) return TF_ERR_SIZE;
  if (tf::launch_recurrence_persistent(launch, workspace, workspace_bytes, static_cast<cudaStream_t>(stream)) != 0) {
    const int ls = tf::launch_status();
    return ls != TF_OK ? ls : TF_ERR_LAUNCH;
  }
  return tf::launch_status();
}


const char* tf_status_string(int status) {
  switch (status) {
    case TF_OK: return "ok";
    case TF_ERR_SHAPE: return "L4 recurrence requires state=128, head=64, rotary=32";
    case TF_ERR_ARG: return "invalid argument";
    case TF_ERR_LAYOUT: return "unsupported tensor layout (innermost dimension must be contiguous)";
    case TF_ERR_DEVICE: return "current CUDA device is not an sm_100 (B200) GPU";
    case TF_ERR_LAUNCH: return "CUDA launch failed";
    case TF_ERR_SIZE: return "size exceeds the documented maximum";
    default: return "unknown status";
  }
}

int tf_version(void) { return 100; }

const char* tf_last_cuda_error(void) { return tf::g_last_error; }

int tf_device_error(int reset) { return tf::read_device_error(reset); }

int tf_error_watch_init(void) {
  static std::mutex m;
  std::lock_guard<std::mutex> lock(m);
  if (tf::g_host_error.load()) return TF_OK;
  int* w = nullptr;
  const cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&w), sizeof(int),
                                      cudaHostAllocMapped | cudaHostAllocPortable);
  if (e != cudaSuccess) {
    snprintf(tf::g_last_error, sizeof tf::g_last_error, "%s", cudaGetErrorString(e));
    (void)cudaGetLastError();
    return TF_ERR_DEVICE;
  }
  *reinterpret_cast<volatile int*>(w) = 0;
  tf::g_host_error.store(w);
  return TF_OK;
}

int tf_device_error_pending(void) {
  const int* w = tf::g_host_error.load();
  return w ? *reinterpret_cast<const volatile int*>(w) : 0;
}

int tf_set_flag_wait_ns(long long ns) {
  if (ns < 0) return TF_ERR_ARG;
  tf::g_flag_wait_ns.store(ns == 0 ? 2000000000ull : static_cast<unsigned long long>(ns));
  return TF_OK;
}

size_t tf_recurrence_workspace_size(int batch, int seqlen, int heads) {
  if (batch <= 0 || seqlen <= 0 || heads <= 0) return 0;
  return tf::recurrence_workspace_bytes(batch, seqlen, heads);
}

int tf_fused_mamba_fwd(const void* q, const void* k, const void* v, const float* adt,
                       const float* dt, const void* trap, int trap_dtype, const float* qb,
                       const float* kb, const void* angles, const float* d, const void* z,
                       void* out, const int64_t* strides, int batch, int seqlen, int heads,
                       int groups, void* workspace, size_t workspace_bytes, void* stream) {
  return tf::recurrence_entry(q, k, v, adt, dt, trap, trap_dtype, qb, kb, angles, d, z, out,
                              strides, batch, seqlen, heads, groups, nullptr, nullptr, 1e-5f,
                              nullptr, workspace, workspace_bytes, stream);
}

int tf_mamba_recurrence_fwd_static(const void* q, const void* k, const void* v, const float* adt,
                                   const float* dt, const void* trap, int trap_dtype,
                                   const float* qb, const float* kb, const void* angles,
                                   const float* d, const void* z, void* out,
                                   const int64_t* strides, int batch, int seqlen, int heads,
                                   int groups, const float* q_norm_w, const float* k_norm_w,
                                   float eps, const int64_t* lengths, void* stream) {
  // Everything is validated before the shared array is touched: a rejected call
  // leaves its contents as they were.
  tf::RecurrenceParams p;
  bool empty = false;
  int st = tf::recurrence_params(q, k, v, adt, dt, trap, trap_dtype, qb, kb, angles, d, z, out, strides, batch,
                                 seqlen, heads, groups, q_norm_w, k_norm_w, eps, lengths, p, empty);
  if (st != TF_OK || empty) return st;
  if (tf::recurrence_workspace_bytes(batch, seqlen, heads) > tf::static_workspace_capacity()) {
    snprintf(tf::g_last_error, sizeof tf::g_last_error,
             "problem needs %zu workspace bytes; the static workspace holds %zu",
             tf::recurrence_workspace_bytes(batch, seqlen, heads), tf::static_workspace_capacity());
    return TF_ERR_SIZE;
  }
  void* ws = nullptr;
  size_t bytes = 0;
  st = tf::prepare_static_workspace(batch, seqlen, heads, static_cast<cudaStream_t>(stream), &ws, &bytes);
  if (st != TF_OK) return st;
  return tf::recurrence_launch(p, ws, bytes, stream);
}

int tf_mamba_recurrence_fwd(const void* q, const void* k, const void* v, const float* adt,
                            const float* dt, const void* trap, int trap_dtype, const float* qb,
                            const float* kb, const void* angles, const float* d, const void* z,
                            void* out, const int64_t* strides, int batch, int seqlen,
                            int heads, int groups, const float* q_norm_w,
                            const float* k_norm_w, float eps, const int64_t* lengths,
                            void* workspace, size_t workspace_bytes, void* stream) {
  return tf::recurrence_entry(q, k, v, adt, dt, trap, trap_dtype, qb, kb, angles, d, z, out,
                              strides, batch, seqlen, heads, groups, q_norm_w, k_norm_w, eps,
                              lengths, workspace, workspace_bytes, stream);
}

}  // extern "C"

// Parameters of the fused Mamba-3 recurrence launch (shared by the kernels and
// the C-ABI launcher).
#pragma once

#include <cuda.h>  // CUtensorMap (a plain 128-byte descriptor; no driver-library linking)

#include "tf_common.cuh"

namespace tf {

struct alignas(64) RecurrenceParams {
  // Set by the launcher when every row of q, k, v, z and the angles is 16-byte
  // aligned with 16-byte strides: the producer stages a unit's rows with these
  // tensor maps (TMA) instead of per-thread cp.async. Boxes of 64 time steps.
  CUtensorMap tm_q, tm_k, tm_v, tm_z, tm_a;
  int tma;

  const bf16* q;       // [B,T,Hq,128]
  const bf16* k;       // [B,T,Hq,128]
  const bf16* v;       // [B,T,H,64]
  const bf16* z;       // [B,T,H,64]
  const bf16* ang;     // [B,T,H,32] raw angle controls
  const float* adt;    // [B,H,T]
  const float* dt;     // [B,H,T]
  const void* trap;    // [B,H,T] f32 or bf16, pre-sigmoid
  const float* qb;     // [H,128]
  const float* kb;     // [H,128]
  const float* d;      // [H]
  const float* qw;     // [128] C_norm weight, or null
  const float* kw;     // [128] B_norm weight, or null
  const int64_t* lengths;  // [B] or null
  bf16* out;           // [B,T,H,64]
  int64_t sq[4], sk[4], sv[4], sz[4], sa[4], so[4];
  int64_t sadt[3], sdt[3], str[3];
  float eps;
  int trap_bf16;
  int B, T, H, Hq;
  // Raw controls (mamba.py:58-63 computed in the producer instead of adt/dt):
  // a, ddt [B,T,H] BF16 views of the projection, dt_bias [H], A floor.
  const bf16* a_raw;
  const bf16* ddt_raw;
  int64_t sar[3], sdr[3];
  const float* dt_bias;
  float a_floor;
  int raw_controls;
  // Reverse: local step t of a row reads and writes time len-1-t (the backward
  // direction of the bidirectional pair, model.py:175-179, without the copies).
  int reverse;
  // Set by the launcher: angle rows are 8-byte aligned with contiguous pairs
  // (staged by cp.async with the other rows).
  int ang_vec;
  // Set by the launcher: how long a wait on another CTA's chunk flag may last
  // before the kernel gives up (records an error and carries on), and the
  // host-mapped error word it then also sets (null when none is set up).
  unsigned long long flag_wait_ns;
  int* err_host;
  // Set by the launcher: element extent (largest offset + 1) of each tensor the
  // kernel reads or writes, and the workspace's unit count. A build with
  // TF_DEBUG_BOUNDS checks every global access of the kernel against them.
  int64_t ext_q, ext_k, ext_v, ext_z, ext_a, ext_out, ext_dt, ext_adt, ext_trap, ext_ar, ext_dr;
};

// One launch may run up to two directions over the same (B, T, H) shape; their
// units share the ticket space (chunk-major, then direction).
struct RecurrenceLaunch {
  RecurrenceParams dir[2];
  int ndir;
};

// Persistent chunk-parallel tensor-core kernel (any T). `workspace` must hold
// recurrence_workspace_bytes(B, T, H) bytes, zero-filled before its first use
// and then reused unchanged. Returns 0 on success.
size_t recurrence_workspace_bytes(int B, int T, int H, int ndir = 1);
int launch_recurrence_persistent(const RecurrenceLaunch& launch, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream);
// Device error word set when a kernel's bounded wait gave up (synchronous read).
int read_device_error(int reset);
// Host-mapped copy of the error word (readable without a synchronisation), the
// flag-wait limit applied to later launches, and their set-up (tf_api.cu).
int* host_error_word();
unsigned long long flag_wait_limit_ns();
// The library's own workspace array (see recurrence_persistent.cu): capacity,
// and per-call preparation (device-address set-up on first use, clearing).
size_t static_workspace_capacity();
int prepare_static_workspace(int B, int T, int H, cudaStream_t stream, void** ws, size_t* bytes);

}  // namespace tf

/*
 * trifusion_b200 — C ABI of the B200 (sm_100a) kernels for the fused Mamba-3
 * recurrence hot path of TriFusion-FP (reference: tlstngud/TriFusion-FP-Kernel
 * 0.1.0, Python package `trifusion_l4`).
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * launches on the given CUDA stream (a `cudaStream_t` passed as `void*`; NULL
 * is the legacy default stream), never synchronises, never allocates device
 * memory, and returns a tf_status code. The library keeps no mutable host
 * state besides a per-device attribute cache filled on first use, so the calls
 * can be captured in CUDA graphs once each device has seen one call.
 *
 * Workspace. The recurrence kernels exchange chunk states through a caller-
 * owned device workspace (size from tf_recurrence_workspace_size). It must be
 * zero-filled once before its first use and then passed back unchanged: the
 * kernels leave it ready for the next launch themselves (launch-epoch tags, no
 * clearing). Launches that share a workspace must not overlap in time; give
 * each concurrently running stream its own workspace.
 *
 * Strides are in ELEMENTS, in the order of the reference tensor's dimensions.
 * BF16 tensors are raw 16-bit bfloat16 values.
 */
#ifndef TRIFUSION_B200_H
#define TRIFUSION_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. The Python host layer maps TF_ERR_SHAPE to ValueError with
 * the reference message (mamba_fused.py:160) and the rest to RuntimeError. */
enum tf_status {
  TF_OK = 0,
  TF_ERR_SHAPE = 1,    /* q/k width != 128, head != 64 or rotary != 32 */
  TF_ERR_ARG = 2,      /* null pointer, non-positive size, H % Hq != 0, bad dtype */
  TF_ERR_LAYOUT = 3,   /* a stride/alignment the kernels cannot address */
  TF_ERR_DEVICE = 4,   /* current device is not sm_100 */
  TF_ERR_LAUNCH = 5,   /* CUDA launch error (cudaGetLastError) */
  TF_ERR_SIZE = 6      /* a size beyond a documented maximum */
};

enum tf_dtype { TF_F32 = 0, TF_BF16 = 1 };

/* Human-readable text of a status code (static storage). */
const char* tf_status_string(int status);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int tf_version(void);

/* Last CUDA error string recorded by this thread (static storage). */
const char* tf_last_cuda_error(void);

/* Device-side error word of the current device: non-zero after a kernel's
 * bounded wait on the tensor core gave up (the kernel then returns instead of
 * hanging). Synchronous; `reset` != 0 clears it. */
int tf_device_error(int reset);

/* Bytes of workspace the recurrence needs for [batch, seqlen, heads]
 * (0 for an empty problem). */
size_t tf_recurrence_workspace_size(int batch, int seqlen, int heads);

/* ------------------------------------------------------------------------
 * Fused Mamba-3 SISO recurrence — drop-in for
 *   trifusion_l4.mamba_fused.fused_mamba(q, k, v, adt, dt, trap, qb, kb,
 *                                        angles, d, z)      (mamba_fused.py:155-191)
 * and its kernel `_fused` (mamba_fused.py:17-152).
 *
 *   q, k    [B,T,Hq,128] bf16       v, z  [B,T,H,64] bf16
 *   adt, dt [B,H,T] f32             trap  [B,H,T] f32 or bf16 (trap_dtype), pre-sigmoid
 *   qb, kb  [H,128] f32 contiguous  angles [B,T,H,32] bf16 raw (head stride may be 0)
 *   d       [H] f32                 out   [B,T,H,64] bf16 (caller-allocated)
 *
 * `strides` holds 33 int64 element strides in this order:
 *   q[4] k[4] v[4] adt[3] dt[3] trap[3] angles[4] z[4] out[4]
 * The last dimension of every bf16 tensor must have stride 1.
 * ------------------------------------------------------------------------ */
int tf_fused_mamba_fwd(const void* q, const void* k, const void* v,
                       const float* adt, const float* dt, const void* trap, int trap_dtype,
                       const float* qb, const float* kb, const void* angles,
                       const float* d, const void* z, void* out,
                       const int64_t* strides, int batch, int seqlen, int heads,
                       int groups, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * The same recurrence with the work around it fused in (no counterpart as one
 * call in the reference; it replaces this sequence of reference launches):
 *   - q_norm_w / k_norm_w (nullable, [128] f32): C_norm/B_norm RMSNorm of the
 *     raw q/k rows before the bias (mamba.py:56-57 -> kernels/native.py:8-39,69),
 *     FP32 statistics, result rounded to bf16 like the reference's norm output;
 *   - lengths (nullable, [B] int64): rows t >= lengths[b] of `out` are written
 *     as zeros (the length mask model.py:174, primitives.py:65-70), and the
 *     recurrence stops at lengths[b] since later rows cannot reach earlier ones.
 * `eps` is the RMSNorm epsilon (1e-5 in the reference).
 * ------------------------------------------------------------------------ */
int tf_mamba_recurrence_fwd(const void* q, const void* k, const void* v,
                            const float* adt, const float* dt, const void* trap,
                            int trap_dtype, const float* qb, const float* kb,
                            const void* angles, const float* d, const void* z, void* out,
                            const int64_t* strides, int batch, int seqlen, int heads,
                            int groups, const float* q_norm_w, const float* k_norm_w,
                            float eps, const int64_t* lengths, void* workspace,
                            size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------
 * tf_mamba_recurrence_fwd without a caller workspace; it allocates nothing.
 * No counterpart in the reference (which always allocates through PyTorch).
 *
 * For callers that cannot allocate device memory: plugin hosts that own all
 * GPU memory through their own pool and expose no allocation hook, and
 * latency-critical services that forbid cudaMalloc after start-up. The
 * workspace is a 64 MiB array inside the library, held on every GPU that loads
 * it until exit; problems needing more (tf_recurrence_workspace_size) return
 * TF_ERR_SIZE without launching. The first call on a device sets up that
 * device's array address and must come before any stream capture. Every call
 * clears the array's header and chunk flags on `stream` before the launch;
 * calls that overlap on the GPU share the array and race, so serialise them.
 * Same arguments and results as tf_mamba_recurrence_fwd otherwise.
 * ------------------------------------------------------------------------ */
int tf_mamba_recurrence_fwd_static(const void* q, const void* k, const void* v,
                                   const float* adt, const float* dt, const void* trap,
                                   int trap_dtype, const float* qb, const float* kb,
                                   const void* angles, const float* d, const void* z,
                                   void* out, const int64_t* strides, int batch, int seqlen,
                                   int heads, int groups, const float* q_norm_w,
                                   const float* k_norm_w, float eps, const int64_t* lengths,
                                   void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRIFUSION_B200_H */

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

/* Device-side error word of the current device: non-zero after one of a
 * recurrence kernel's bounded waits gave up (on the tensor core, on the other
 * warps of its CTA, or on another CTA's chunk flag); the kernel then finishes
 * instead of hanging, and the outputs of that launch are invalid. Synchronous;
 * `reset` != 0 clears it (and the host-mapped word below). */
int tf_device_error(int reset);

/* Sets up a pinned, device-mapped host word that the kernels also set when a
 * wait gives up, so the host can poll it without synchronising
 * (tf_device_error_pending). Call once, before any stream capture; allocates
 * host memory only. Launches made before it report to the device word only. */
int tf_error_watch_init(void);

/* The host-mapped error word: non-zero once a launch has given up a wait
 * (asynchronous: it shows after that launch has run). 0 when not set up. */
int tf_device_error_pending(void);

/* Limit, in nanoseconds, of a recurrence kernel's waits on other CTAs' chunk
 * flags in later launches (0 restores the default of 2 s). A diagnostic
 * control: a launch whose wait runs out records the error above and completes
 * with invalid outputs. Waits inside a CTA keep their fixed 2 s limit. */
int tf_set_flag_wait_ns(long long ns);

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
 * device's array address and must come before any stream capture; with lazy
 * module loading the array is reserved then, so make that call at start-up,
 * before a memory pool takes the device's memory (if the array cannot be had
 * the call returns TF_ERR_DEVICE and tf_last_cuda_error names why). Arguments
 * are validated before the array is touched. Every call
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

/* ------------------------------------------------------------------------
 * One launch for one or two recurrences over the same [B, T, H] shape (the
 * forward and backward directions of a block's bidirectional pair,
 * model.py:173-179), each optionally
 *   - computing its controls from the projection views (prologue fusion of
 *     mamba.py:58-63 / kernels/buffers.py:82-101): a_raw, ddt_raw [B,T,H] BF16
 *     with dt = softplus(ddt + dt_bias[h]) and adt = min(-(relu(a) +
 *     1/(1 - min(a, 0))), -a_floor) * dt, instead of adt/dt;
 *   - reading and writing the valid prefix of every row in reverse time order
 *     (`reverse`): local step t uses time len-1-t, so the backward direction
 *     needs no reverse_valid copies (kernels/__init__.py:43-54) around it;
 *     rows at or past the length come out zero in place.
 * q_norm_w/k_norm_w and `lengths` act as in tf_mamba_recurrence_fwd. Strides are
 * the 33 of tf_fused_mamba_fwd followed by a_raw (b, t, h) and ddt_raw (b, t, h).
 * ------------------------------------------------------------------------ */
typedef struct tf_recurrence_io {
  const void* q;
  const void* k;
  const void* v;
  const void* z;
  const void* angles;
  const float* qb;
  const float* kb;
  const float* d;
  const float* adt;       /* [B,H,T] FP32, or NULL when a_raw/ddt_raw are given */
  const float* dt;
  const void* trap;
  int trap_dtype;
  const void* a_raw;      /* [B,T,H] BF16 views, or NULL */
  const void* ddt_raw;
  const float* dt_bias;   /* [H] */
  float a_floor;
  const float* q_norm_w;  /* [128] or NULL */
  const float* k_norm_w;
  void* out;
  int64_t strides[39];
  int reverse;
} tf_recurrence_io;

/* Workspace bytes for `count` (1 or 2) directions of [B, T, H]. */
size_t tf_recurrence_workspace_size_multi(int count, int batch, int seqlen, int heads);

/* Runs io[0..count-1] in one launch; the workspace rules of the header apply.
 * No counterpart function in the reference: it replaces the pair of
 * Mamba3Inference calls with their reverse_valid copies and the controls
 * launches of model.py:175-179 / mamba.py:58-66. */
int tf_mamba_recurrence_multi_fwd(const tf_recurrence_io* io, int count, int batch, int seqlen,
                                  int heads, int groups, float eps, const int64_t* lengths,
                                  void* workspace, size_t workspace_bytes, void* stream);

/* ========================================================================
 * Satellite operators on the recurrence path. Contiguous row-major tensors
 * (the reference wrappers call .contiguous() first); `dtype` is TF_F32 or
 * TF_BF16; arithmetic is FP32 with one rounding to the output type; copy and
 * index operators move raw bits (bit-exact). Lengths are int64 device arrays;
 * values outside [0, T] are clamped to it.
 * ======================================================================== */

/* A6 RMSNorm: y = x * rsqrt(mean(x^2) + eps) * w over rows of `width`; y has
 * x's dtype, w is FP32. Replaces kernels/native.py:69-70 `rms` (its `_norm`
 * MODE 0, native.py:8-39) and RMSNorm.forward (kernels/__init__.py:23-27). */
int tf_rms_fwd(const void* x, int dtype, const float* w, void* y, int64_t rows, int width,
               float eps, void* stream);

/* Evidence norm: rows with mask != 0 take x + value * 2 sigmoid(gate), others 0;
 * then RMSNorm; FP32 out. Replaces kernels/native.py:73-74 `evidence_norm`
 * (`_norm` MODE 1, native.py:28-34). */
int tf_evidence_norm_fwd(const void* x, int x_dtype, const void* value, const void* gate,
                         int vg_dtype, const float* w, const uint8_t* mask, float* y,
                         int64_t rows, int width, float eps, void* stream);

/* A10 mean_norm of the bidirectional pair: y = RMSNorm((a + b) / 2) * w, FP32 out.
 * Replaces kernels/native.py:77-78 `mean_norm` (`_norm` MODE 2, native.py:35-37). */
int tf_mean_norm_fwd(const void* a, const void* b, int dtype, const float* w, float* y,
                     int64_t rows, int width, float eps, void* stream);

/* A7 controls: A = min(-(max(a,0) + 1/(1 - min(a,0))), -a_floor),
 * dt = softplus(ddt + dt_bias[h]) (identity above 20), adt = A * dt; inputs
 * [B,T,H] with strides {a: b,t,h, ddt: b,t,h} (h stride must be 1), outputs
 * [B,H,T] FP32 contiguous. Replaces kernels/buffers.py:82-101 `mamba_controls`
 * (`_controls`, kernels/primitives.py:190-216). */
int tf_mamba_controls_fwd(const void* a, const void* ddt, int dtype, const int64_t* strides,
                          const float* dt_bias, float a_floor, float* adt, float* dt, int batch,
                          int seqlen, int heads, void* stream);

/* A8 fused into the block's residual tail: y[r, :] = mask[r] ? a[r, :] + b[r, :] : 0
 * over rows of `width` (a multiple of 4), a and y FP32, b FP32 or BF16 (added
 * exactly in FP32). Replaces model.py:199 `mask(r + down(f))` (the FP32 add and
 * the `_mask` pass of kernels/buffers.py:6-10) with one pass. */
int tf_masked_add_fwd(const float* a, const void* b, int b_dtype, const uint8_t* mask, float* y, int64_t rows,
                      int width, void* stream);

/* A8 length mask: row r of y = row r of x where mask[r] != 0, else zero bytes.
 * Replaces kernels/buffers.py:6-10 `mask_buffer` (`_mask`, primitives.py:65-70). */
int tf_mask_rows_fwd(const void* x, const uint8_t* mask, void* y, int64_t rows,
                     int64_t row_bytes, void* stream);

/* A9 valid-prefix reversal: y[b,t] = x[b, len-1-t] for t < len, else zero bytes.
 * Replaces kernels/__init__.py:43-54 `reverse_valid` (`_reverse`, primitives.py:40-47). */
int tf_reverse_valid_fwd(const void* x, const int64_t* lengths, void* y, int batch, int seqlen,
                         int64_t row_bytes, void* stream);

/* A11 SwiGLU: x [rows, 2d] -> y[r,c] = silu(x[r,c]) * x[r,d+c], x's dtype.
 * Replaces kernels/__init__.py:30-40 `swiglu` (`_swiglu`, primitives.py:25-37). */
int tf_swiglu_fwd(const void* x, int dtype, void* y, int64_t rows, int d, void* stream);

/* A12 branch gate: x [rows, 3d], gate [rows, 3] -> y[r,j,:] = x[r,j,:] * 2 sigmoid(gate[r,j]).
 * Replaces kernels/__init__.py:57-81 `gated_concat` (`_gate`, primitives.py:50-62). */
int tf_gated_concat_fwd(const void* x, int dtype, const void* gate, int gate_dtype, void* y,
                        int64_t rows, int d, void* stream);

/* A13 Pool4: x [B,T,D] -> y [B,ceil(T/4),D], the mean of the valid frames of each
 * group of 4 (divisor max(min(len - 4g, 4), 1)); bit-identical to the reference
 * kernel. Replaces kernels/buffers.py:35-43 `Pool4.apply` (`_pool4`,
 * primitives.py:90-113) and masking.py:59-69 `Grids.pool`. */
int tf_pool4_fwd(const void* x, int dtype, const int64_t* lengths, void* y, int batch, int seqlen,
                 int width, void* stream);

/* Pool4 with the output type chosen: FP32 x, BF16 y (the FP32 means rounded once,
 * what autocast passes to the attention's qkv projection, model.py:127-129). */
int tf_pool4_out_fwd(const void* x, int dtype, const int64_t* lengths, void* y, int y_dtype, int batch, int seqlen,
                     int width, void* stream);

/* A13 masked time mean: y[b,:] = sum_{t<len} x[b,t,:] / len, FP32 [B,D].
 * Replaces decoder.py:60-62 (`(x.float() * mask).sum(1) / lengths`). */
int tf_masked_mean_fwd(const void* x, int dtype, const int64_t* lengths, float* y, int batch,
                       int seqlen, int width, void* stream);

/* Decoder query read: 10 queries x 8 heads of width 32 (q [10, 256] BF16, head c at
 * columns 32c) attend in FP32 over keys and values read from the BF16 projection rows
 * kv [batch, time, >= 512] (row pitch kv_pitch elements, a multiple of 8, base 16-byte
 * aligned; k of head c at column 32c, v at 256 + 32c); key j is valid when
 * j < min(time, lengths[b] * keys_per_length). y [batch, 10, 256] BF16 (row i holds the
 * 8 heads' outputs side by side); a row with no valid key is NaN, like the reference's
 * softmax. `state` is FP32 scratch of tf_query_read_state_floats(batch, time) floats.
 * Replaces decoder.py:26-30 (the kv permute, q expand, attention.py:8-18
 * `masked_attention` and the transpose/reshape before `out`); equal to it up to FP32
 * summation order. */
int64_t tf_query_read_state_floats(int batch, int time);
int tf_query_read_fwd(const void* q, const void* kv, int64_t kv_pitch, const int64_t* lengths, int keys_per_length,
                      float* state, int64_t state_floats, void* y, int batch, int time, void* stream);

/* A13 end gather: y[b] = x[b, len-1] (len = 0 reads row T-1, like PyTorch's -1 index).
 * Replaces decoder.py:63 (`mf[arange(b), lengths - 1]`). */
int tf_end_gather_fwd(const void* x, const int64_t* lengths, void* y, int batch, int seqlen,
                      int64_t row_bytes, void* stream);

/* Local evidence of the decoder: for each clip b and class c in {0, 1}, the scores
 * float(local[b, t, c]) with frames t >= fine_lengths[b] at -inf, their k = min(25, time)
 * largest (ties at the k-th value resolve to the earliest frames), and
 * top[b, c, :] = sum over the first min(fine_lengths[b], k) picks of float(features[b, t, :])
 * divided by that count (NaN when it is 0, like the reference). `local` BF16 rows of pitch
 * local_pitch elements (classes in columns 0 and 1), `features` BF16 rows of pitch
 * feat_pitch (256 used), both [batch, time, pitch] contiguous over rows; writes
 * local_f32 [batch, time, 2] (the FP32 copy of `local`) and top [batch, 2, 256] FP32.
 * time <= 12288 (else TF_ERR_SIZE). Replaces decoder.py:65-76 (`local.float()`, the
 * masked_fill, topk, gather and masked mean); the selection is exact, the mean equal up
 * to FP32 summation order. */
int tf_local_topk_fwd(const void* local, int64_t local_pitch, const void* features, int64_t feat_pitch,
                      const int64_t* fine_lengths, float* local_f32, float* top, int batch, int time,
                      void* stream);

/* Decoder heads: voice = silu(voice_lat(cat(deep_q[0], fine_q[0], global, top[:, 0], memory))),
 * music likewise (query group 1, top[:, 1]), file = silu(file_head[0](cat(deep_q[2], fine_q[2],
 * global, memory, voice, music))), and logits [batch, 5] FP32 = [f, v0, m0, v1, m1] with
 * v = voice_head(voice), m = music_head(music), f = file_head[2](file). deep_rows and
 * fine_rows are the query reads' BF16 out-projection rows [batch, 10, 256]; deep_q[g] and
 * fine_q[g] are their group means over rows 0-3, 4-7 and 8-9 (rounded once to BF16);
 * global_feature and memory are BF16 [batch, 256], top FP32 [batch, 2, 256] (rounded to
 * BF16 as autocast does for the concatenation), all contiguous and 16-byte aligned
 * (else TF_ERR_LAYOUT). Weights are the BF16 Linear weights
 * ([out, in] row-major, 16-byte aligned) and biases: voice/music lat [256, 1280] + [256],
 * voice/music head [2, 256] + [2], file_head[0] [256, 1536] + [256], file_head[2] [1, 256] + [1].
 * Every projection accumulates in FP32, adds the bias and rounds to BF16; SiLU rounds again.
 * `scratch` holds tf_decoder_heads_scratch_bytes(batch) bytes (16-byte aligned). Three
 * launches. Replaces decoder.py:77-89 (five concatenations, five projections, two SiLUs,
 * the logits concatenation and cast); equal to the reference up to FP32 summation order. */
int64_t tf_decoder_heads_scratch_bytes(int batch);
int tf_decoder_heads_fwd(const void* deep_rows, const void* fine_rows, const void* global_feature,
                         const void* memory, const float* top, const void* w_voice, const void* b_voice,
                         const void* w_music, const void* b_music, const void* w_vhead, const void* b_vhead,
                         const void* w_mhead, const void* b_mhead, const void* w_file1, const void* b_file1,
                         const void* w_file2, const void* b_file2, void* scratch, int64_t scratch_bytes,
                         float* logits, int batch, void* stream);

/* RMSNorm as tf_rms_fwd with the output type chosen (`y_dtype` TF_F32 or TF_BF16):
 * a BF16 result is the FP32 result rounded once, i.e. what autocast would feed the
 * next projection. Replaces `RMSNorm` (kernels/__init__.py:23-27) followed by the
 * autocast cast of its output before model.py:198 `gate_up`. */
int tf_rms_out_fwd(const void* x, int dtype, const float* w, void* y, int y_dtype, int64_t rows, int width,
                   float eps, void* stream);

/* Residual add and RMSNorm in one pass: sum = x + a (FP32; a FP32 or BF16, added
 * exactly) written to `sum`, y = rms(sum) * w in `y_dtype` (rounded once).
 * Replaces model.py:197-198 (`r = x + merge(...)`, then `ff_norm(r)` and autocast's
 * cast before gate_up). width % 4 == 0, `sum` 16-byte aligned. */
int tf_add_rms_fwd(const float* x, const void* a, int a_dtype, const float* w, float* sum, void* y, int y_dtype,
                   int64_t rows, int width, float eps, void* stream);

/* RMSNorm as tf_rms_out_fwd, written into the slice of a wider row: output row r
 * starts at y + r * y_pitch (elements, >= width). With `y2` non-NULL the same
 * values are also written, rounded once to BF16, at y2 + r * y2_pitch. Replaces
 * model.py:159-161 (`cn`, `an`, then `torch.cat((cn, an))` for e_down): each norm
 * writes its half of e_down's input row and its third of the gate's BF16 input
 * row directly. */
int tf_rms_pitched_fwd(const void* x, int dtype, const float* w, void* y, int y_dtype, int64_t y_pitch,
                       void* y2, int64_t y2_pitch, int64_t rows, int width, float eps, void* stream);

/* mean_norm (tf_mean_norm_fwd, FP32 y [rows, width]) that also writes y rounded
 * once to BF16 at y2 + r * y2_pitch: the middle third of the gate's input row,
 * which model.py:185-186 forms as `torch.cat((cn, mn, an))` cast by autocast. */
int tf_mean_norm_copy_fwd(const void* a, const void* b, int dtype, const float* w, float* y, void* y2,
                          int64_t y2_pitch, int64_t rows, int width, float eps, void* stream);

/* Branch gate (tf_gated_concat_fwd) over three separate branch tensors instead of
 * their concatenation: branch 0 at x0 + r * pitches[0], branch 1 (FP32) at
 * x1 + r * pitches[1], branch 2 at x2 + r * pitches[2]; x0/x2 of type `dtype`;
 * y [rows, 3d] FP32. Bit-equal to tf_gated_concat_fwd on the FP32 concatenation.
 * Replaces model.py:185-186 `gated_concat(torch.cat((cn, mn, an)), gate)`. */
int tf_gated_branches_fwd(const void* x0, const float* x1, const void* x2, int dtype, const int64_t* pitches,
                          const void* gate, int gate_dtype, float* y, int64_t rows, int d, void* stream);

/* Branch gate with its three-output projection, one warp per row: from the BF16
 * gate-input row s (width 3d, rows every s_pitch elements), g_j = bf16(s . w[j] +
 * bias[j]) with FP32 products and sums (w [3, 3d] BF16, bias [3] BF16 or NULL),
 * then y[r, j, :] = x_j * 2 sigmoid(g_j) into FP32 y [rows, 3d], with branches 0
 * and 2 read from s and branch 1 from the FP32 rows x1 (x1_pitch). g [rows, 3]
 * BF16 receives the gate values when non-NULL. d % 4 == 0, s/w 8-byte and x1/y
 * 16-byte aligned, pitches multiples of 4 (else TF_ERR_LAYOUT). Replaces
 * model.py:185-186 `gated_concat(s, self.gate(s))` under BF16 autocast (the
 * nn.Linear(3d, 3) GEMM and kernels/__init__.py:57-81); g equals the GEMM's
 * output up to FP32 summation order. */
int tf_gate_branches_fwd(const void* s, int64_t s_pitch, const float* x1, int64_t x1_pitch, const void* w,
                         const void* bias, float* y, void* g, int64_t rows, int d, void* stream);

/* RMSNorm then SiLU: a = rms(x) * w rounded to x's type, y = a / (1 + e^-a) (PyTorch's
 * silu on the norm's output tensor); y has x's type. Replaces model.py:120
 * `F.silu(self.norm(h))` (RMSNorm of kernels/__init__.py:23-27 and the SiLU). */
int tf_rms_silu_fwd(const void* x, int dtype, const float* w, void* y, int64_t rows, int width, float eps,
                    void* stream);

/* Evidence norm as tf_evidence_norm_fwd with the output type chosen (TF_F32 or
 * TF_BF16, the FP32 result rounded once). Replaces native.py:73-74 followed by the
 * autocast cast before the Mamba in_proj (mamba.py:42). */
int tf_evidence_norm_out_fwd(const void* x, int x_dtype, const void* value, const void* gate, int vg_dtype,
                             const float* w, const uint8_t* mask, void* y, int y_dtype, int64_t rows, int width,
                             float eps, void* stream);

/* Evidence norm as tf_evidence_norm_out_fwd with `value` and `gate` rows every
 * vg_pitch elements (>= width), e.g. the two halves of one stacked projection row
 * [rows, 2 * width]. Replaces native.py:73-74 fed by model.py:163-166's two
 * projections `e_value(z)`, `e_gate(z)` (here one GEMM over both weights). */
int tf_evidence_norm_pitched_fwd(const void* x, int x_dtype, const void* value, const void* gate, int vg_dtype,
                                 int64_t vg_pitch, const float* w, const uint8_t* mask, void* y, int y_dtype,
                                 int64_t rows, int width, float eps, void* stream);

/* Depthwise Conv1d over time on [B, T, C] rows with zero padding outside [0, T):
 * y[b,t,c] = t < lengths[b] ? sum_k x[b, t+k-K/2, c] w[c,k] + bias[c] : 0, inputs
 * rounded to BF16, BF16 out; w [C, K] and bias [C] (may be NULL) BF16; K in
 * {3, 5, 7}; C % 4 == 0. Replaces kernels/buffers.py:13-32 `depthwise_masked`
 * (`_dw_forward`, kernels/primitives.py:73-87), used by model.py:70-72,186-190. */
int tf_depthwise_masked_fwd(const void* x, int dtype, const void* w, const void* bias,
                            const int64_t* lengths, void* y, int batch, int seqlen, int channels,
                            int taps, void* stream);

/* As tf_depthwise_masked_fwd, plus the input itself: y = bf16(x + bf16(conv(x))),
 * the sum in FP32. Replaces model.py:188-189 (`v + depthwise_masked(v)` rounded by
 * autocast before the merge projection). */
int tf_depthwise_residual_fwd(const void* x, int dtype, const void* w, const void* bias, const int64_t* lengths,
                              void* y, int batch, int seqlen, int channels, int taps, void* stream);

/* As tf_depthwise_masked_fwd on the GLU of x: x [batch, seqlen, 2 * channels] BF16 (the
 * local branch's up projection, 8-byte aligned), conv input h = bf16(a * (1 / (1 + e^-g)))
 * with a = x[.., c], g = x[.., channels + c] (PyTorch's glu on a BF16 tensor), output
 * BF16 [batch, seqlen, channels]. Replaces model.py:122 `F.glu(self.up(x))` and the
 * depthwise conv that reads its result (model.py:123-124); bit-exact against the two. */
int tf_glu_depthwise_fwd(const void* x, const void* w, const void* bias, const int64_t* lengths, void* y,
                         int batch, int seqlen, int channels, int taps, void* stream);

/* Rotary q/k of the attention branch: x [B, T, 3, H, D] BF16 (the qkv projection)
 * -> y [3, B, H, T, D] FP32 holding BF16-rounded values; q and k pairs rotated by
 * the table angle (cosv/sinv [T, D/2] FP32), v copied. Replaces
 * kernels/buffers.py:46-55 `RotaryQKV.apply` (`_rotary_qkv`,
 * kernels/primitives.py:116-150) and the FP32 widening of attention.py:14-16. */
int tf_rotary_qkv_fwd(const void* x, const float* cosv, const float* sinv, float* y, int batch,
                      int time, int heads, int head_dim, void* stream);

/* Rotary q/k and FP32 masked attention over the pooled rows in one kernel: x
 * [B, LT, 3, H, 64] BF16 (the qkv projection); q and k rotated as tf_rotary_qkv_fwd
 * (cosv/sinv [>= LT, 32] FP32) and rounded to BF16, v as is; key j valid when
 * j < lengths[b]; scores scaled by 1/8, softmax and sums in FP32. y [B, LT, H*64]
 * BF16 (the heads side by side, the out projection's input rows); a row with no
 * valid key is NaN, like the reference's softmax. head_dim must be 64. Replaces
 * model.py:127-133 after `qkv` (kernels/buffers.py:46-55 `RotaryQKV.apply`,
 * attention.py:8-18 `masked_attention`, the transpose/reshape before `out`); equal
 * to it up to FP32 summation order. */
int tf_pooled_attention_fwd(const void* x, const float* cosv, const float* sinv, const int64_t* lengths, void* y,
                            int batch, int low_time, int heads, int head_dim, void* stream);

/* Interpolation from the pooled grid: y[b, t] = t < lengths[b] ?
 * a + (z - a) alpha[b, t] : 0 with a = low[b, left[b, t]], z = low[b, right[b, t]];
 * low [B, LT, D] BF16, y [B, T, D] BF16, D % 4 == 0. Replaces
 * kernels/native.py:119-138 `interpolate` (`_interpolate`, native.py:103-117) and
 * masking.py:71-80 `Grids.interpolate`. */
int tf_interpolate_fwd(const void* low, const int64_t* left, const int64_t* right, const float* alpha,
                       const int64_t* lengths, void* y, int batch, int time, int low_time, int width,
                       void* stream);

/* ------------------------------------------------------------------------
 * Spectrogram front end, on channels-last activations: a [B, C, T, F] tensor
 * stored as [B, T, F, C] (every (b, t, f) position one contiguous row of C).
 * ------------------------------------------------------------------------ */

/* Channel RMSNorm of every (b, t, f) row, zero where t >= lengths[b], then SiLU
 * when `silu` != 0 (the normalised value is rounded to `dtype` first); C <= 256.
 * Replaces kernels/buffers.py:58-79 `front_norm` (`_front_norm`,
 * kernels/primitives.py:153-187), used by front.py:19-43. */
int tf_front_norm_fwd(const void* x, int dtype, const float* w, const int64_t* lengths, void* y,
                      int batch, int time, int freq, int channels, float eps, int silu, void* stream);

/* Stem of the first CNN stage (C_in = 1, C_out = 32, time stride 1): from the
 * [B, T, F] FP32 spectrogram, the 3x3 convolution (stride (1, 2), padding 1;
 * w1 [32, 1, 3, 3] FP32) and the 1x1 skip (stride (1, 2); ws [32] FP32), both as
 * BF16 autocast convolutions (operands rounded to BF16, FP32 accumulation), and
 * the conv branch's masked channel RMSNorm (norm_w [32]) and SiLU; writes
 * h and skip, [B, T, (F-1)/2+1, 32] BF16 channels-last, 16-byte aligned.
 * Replaces front.py:21,33,43 (`self.conv1(x)`, `front_norm(h, ..., silu=True)` of
 * kernels/buffers.py:58-79, `self.skip(x)`) for the first stage (front.py:53);
 * the convolution sums may differ from cuDNN's in summation order (one BF16
 * rounding at most). */
int tf_front_stem_fwd(const float* x, const float* w1, const float* ws, const float* norm_w,
                      const int64_t* lengths, void* h, void* skip, int batch, int time, int freq, float eps,
                      void* stream);

/* Residual tail of a CNN stage: y = t < lengths[b] ? silu(h + skip) : 0, the sum
 * rounded to `dtype` before SiLU. Replaces front.py:43
 * (`clean(F.silu(h + clean(self.skip(x))))`). */
int tf_front_residual_fwd(const void* h, const void* skip, int dtype, const int64_t* lengths, void* y,
                          int batch, int time, int freq, int channels, void* stream);

/* Frequency bands: x [B, T, F, C] -> y [B, T, 8, C], band i the mean over
 * f in [floor(i F / 8), ceil((i + 1) F / 8)). Replaces kernels/native.py:141-163
 * `bands` and front.py:80-87 (adaptive_avg_pool2d + permute). */
int tf_bands_fwd(const void* x, int dtype, void* y, int batch, int time, int freq, int channels,
                 void* stream);

/* Valid-row transfer between padded device tensors and a packed buffer (raw
 * bytes, either direction). No counterpart kernel in the reference, which
 * copies whole padded tensors to the device (audio.py:52-66 pads every batch to
 * its longest clip); rows at or past a clip's length carry nothing the
 * recurrence reads, so a host-fed pipeline moves only the valid ones.
 * Tensor i is `dense[i]`, laid out [batch][groups[i]][steps[i]][step_bytes[i]]
 * contiguously; `lengths` (device, int64 [batch]) gives each clip's valid
 * steps (clamped to [0, steps[i]]). The packed buffer holds, tensor after
 * tensor, for each clip b and group g the valid steps of (b, g) back to back;
 * each tensor's region starts at a 16-byte-aligned offset. `to_dense` = 1
 * copies packed -> dense (the padding rows are left as they are), 0 copies
 * dense -> packed. At most 16 tensors and 65535 clips per call. */
int tf_ragged_copy_fwd(void* packed, void* const* dense, const int64_t* groups, const int64_t* steps,
                       const int64_t* step_bytes, int ntensors, const int64_t* lengths, int batch,
                       int to_dense, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRIFUSION_B200_H */

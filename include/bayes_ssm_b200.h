/*
 * bayes_ssm_b200.h -- C ABI of the B200 (sm_100a) Bayesian-layer kernels.
 *
 * Plain pointers and sizes only.  Every entry point:
 *   - takes device pointers (CUDA global memory of the current device) for
 *     tensors and a cudaStream_t passed as void*; it only enqueues work on
 *     that stream (no host synchronisation, no allocation);
 *   - returns BSSM_OK (0) or a BSSM_ERR_* code; bssm_last_error() then
 *     returns a message for the calling thread.
 *
 * Shapes (row-major, contiguous; N independent chains, T tokens):
 *   keys, queries [N,T,D]; values [N,T,M]; decay [N,T,D]; process,
 *   observation [N,T]; mean0 [N,D,M]; cov0 [N,D,D];
 *   out [N,T,M]; mean_final [N,D,M]; cov_final [N,D,D];
 *   boundary_mean [N,NB+1,D,M]; boundary_cov [N,NB+1,D,D], NB = ceil(T/chunks).
 * Supported (D, M): (1,8), (2,8), (4,8), (8,8) and (64,64).
 * io_dtype selects the element type of keys/values/queries and of their
 * gradients: BSSM_F32 or BSSM_BF16 ((64,64): BSSM_F32 only, as in the
 * reference).  Everything else is float32; the mean, covariance and every
 * reduction are float32.  (64,64) needs no replay states (its backward
 * recomputes each chunk into the workspace, bssm_backward_workspace_bytes).
 *
 * Pointer alignment: every tensor pointer of the recurrence entry points must
 * be 16-byte aligned (any fresh CUDA allocation is); BSSM_ERR_ALIGNMENT
 * otherwise.
 *
 * Reference interface these replace (paths within catid/bayes-ssm): the
 * per-key-dim pybind modules loaded by bayes_ssm/fused_cuda.py:23-55, whose
 * exports are listed at bayes_ssm/persistent_bayes_chunked_d8.cu:653,
 * _d4m8.cu:577, _d2m8.cu:602 and _d1m8.cu:673.
 */
#ifndef BAYES_SSM_B200_H
#define BAYES_SSM_B200_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BSSM_OK 0
#define BSSM_ERR_INVALID 1     /* bad shape, size or null pointer */
#define BSSM_ERR_UNSUPPORTED 2 /* (D, M) or dtype without a kernel */
#define BSSM_ERR_ALIGNMENT 3   /* a vector-loaded pointer is misaligned */
#define BSSM_ERR_CUDA 4        /* CUDA launch or runtime error */
#define BSSM_ERR_WORKSPACE 5   /* workspace missing or too small */
#define BSSM_ERR_TIMEOUT 6     /* a bounded in-kernel wait gave up (bssm_stream_status) */

#define BSSM_F32 0
#define BSSM_BF16 1
#define BSSM_F16 2 /* bssm_check_values only */

/* Message for the last failing call on this thread ("" after success). */
const char *bssm_last_error(void);

/* ABI version: major * 10000 + minor * 100 + patch. */
int bssm_version(void);

/* ---------------------------------------------------------------------
 * Generic entry points.
 * ------------------------------------------------------------------- */

/*
 * Chunked forward: readouts, final state and the chunk-boundary states the
 * backward replays from.  fixed != 0 ignores decay/process/observation (may
 * be NULL) and uses A = 0.97 I, Q = 0.1 I, R = 1.  mean0 == NULL means zeros,
 * cov0 == NULL means identity.  The covariance enters as (cov0 + cov0^T)/2.
 * replay_states (optional, may be NULL): the replay buffer,
 * bssm_replay_states_bytes(...) bytes.  When given, the forward also saves
 * the state at every 4-token boundary inside each chunk and every token's
 * gain u, 1/s and s; a backward given the same buffer replays from them
 * instead of recomputing the chunk (and its thread-per-chain form replays
 * the mean from the saved gains).  The layout is internal to the library.
 * Replaces forward_chunked / forward_chunked_fixed,
 * bayes_ssm/persistent_bayes_chunked_d8.cu:530-548.
 */
int bssm_forward_chunked_ex(int key_dim, int value_dim, int io_dtype, int fixed,
                            const void *keys, const void *values, const void *queries,
                            const float *decay, const float *process, const float *observation,
                            const float *mean0, const float *cov0,
                            float *out, float *mean_final, float *cov_final,
                            float *boundary_mean, float *boundary_cov,
                            float *replay_states, size_t replay_states_bytes,
                            long n, long t, int chunks, double denominator_floor,
                            void *stream);

/* Bytes of the optional replay-state buffer (0 when chunks <= 4: nothing to save). */
size_t bssm_replay_states_bytes(int key_dim, int value_dim, long n, long t, int chunks);

/* Bytes of device workspace bssm_backward_chunked_ex needs (0 allowed). */
size_t bssm_backward_workspace_bytes(int key_dim, int value_dim, long n, long t, int chunks);

/*
 * Chunk-replay backward.  One launch: for every chain, chunks are replayed
 * from boundary_mean/boundary_cov in reverse order and the adjoint runs over
 * each replayed span in the same kernel.
 *   grad_out [N,T,M] (NULL = zeros), grad_mean_final [N,D,M] (NULL = zeros),
 *   grad_cov_final [N,D,D] (NULL = zeros).
 * Outputs grad_keys/grad_values/grad_queries are always written.
 * need_dynamics != 0 also writes grad_decay [N,T,D], grad_process and
 * grad_observation [N,T] (zeros when fixed != 0).
 * need_initial != 0 also writes grad_mean0 [N,D,M] and grad_cov0 [N,D,D]
 * (symmetric: the covariance entered as (cov0 + cov0^T)/2).
 * replay_states: the buffer the forward filled (then no workspace is
 * needed), or NULL.
 * workspace: device memory of bssm_backward_workspace_bytes(...) bytes when
 * replay_states is NULL (NULL allowed when that size is 0).
 * Replaces backward_chunked and its lean / fixed / noinitial variants,
 * bayes_ssm/persistent_bayes_chunked_d8.cu:550-651,
 * bayes_ssm/persistent_bayes_chunked_d2m8.cu:576-600.
 */
int bssm_backward_chunked_ex(int key_dim, int value_dim, int io_dtype, int fixed,
                             int need_dynamics, int need_initial,
                             const void *keys, const void *values, const void *queries,
                             const float *decay, const float *process, const float *observation,
                             const float *mean0, const float *cov0,
                             const float *boundary_mean, const float *boundary_cov,
                             const float *replay_states, size_t replay_states_bytes,
                             const float *grad_out, const float *grad_mean_final,
                             const float *grad_cov_final,
                             void *grad_keys, void *grad_values, void *grad_queries,
                             float *grad_decay, float *grad_process, float *grad_observation,
                             float *grad_mean0, float *grad_cov0,
                             void *workspace, size_t workspace_bytes,
                             long n, long t, int chunks, double denominator_floor,
                             void *stream);

/*
 * Static associative scan (A = I, Q = 0), forward only, float32.
 *   keys/queries [N,T,D], values [N,T,M], observation [N,T] (every entry
 *   finite and >= denominator_floor; the caller validates, the kernel also
 *   flags), mean0 [N,D,M] (NULL = 0), cov0 [N,D,D] (NULL = I; must be
 *   positive definite), out [N,T,M], mean_final [N,D,M], cov_final [N,D,D].
 *   status: device int the caller zeroes; the kernel ORs 1 when a precision
 *   matrix is not positive definite and 2 when an observation variance is
 *   below the floor or not finite.
 * Limits: 1 <= D <= 32, 1 <= M <= 256, N <= 65535 per call.
 * Replaces associative_static_bayesian_cuda, bayes_ssm/replay_ssm.py:276-339
 * (whose default path is the eager information-form scan :155-270).
 */
int bssm_assoc_scan_ex(int key_dim, int value_dim, const float *keys, const float *values,
                       const float *queries, const float *observation, const float *mean0,
                       const float *cov0, float *out, float *mean_final, float *cov_final,
                       int *status, long n, long t, double denominator_floor, void *stream);

/* ---------------------------------------------------------------------
 * Reference-named float32 entry points, one set per key dimension
 * (M = 8; M = 64 for the D = 64 set).  Same arguments as the reference's
 * pybind functions, with the output buffers and the backward workspace
 * supplied by the caller.  The D = 64 set replaces the exports of
 * bayes_ssm/persistent_bayes_chunked.cu:436.
 * ------------------------------------------------------------------- */
#define BSSM_DECLARE_DIM(DN)                                                                     \
    /* forward_chunked: persistent_bayes_chunked_d8.cu:530 and its D4/D2/D1 twins */            \
    int bssm_d##DN##_forward_chunked(const float *keys, const float *values, const float *queries, \
                                     const float *decay, const float *process,                  \
                                     const float *observation, const float *mean0,              \
                                     const float *cov0, float *out, float *mean_final,          \
                                     float *cov_final, float *boundary_mean,                    \
                                     float *boundary_cov, long n, long t, int chunks,           \
                                     double denominator_floor, void *stream);                   \
    /* forward_chunked_fixed: persistent_bayes_chunked_d8.cu:539 */                              \
    int bssm_d##DN##_forward_chunked_fixed(const float *keys, const float *values,               \
                                           const float *queries, const float *decay,            \
                                           const float *process, const float *observation,      \
                                           const float *mean0, const float *cov0, float *out,   \
                                           float *mean_final, float *cov_final,                 \
                                           float *boundary_mean, float *boundary_cov, long n,   \
                                           long t, int chunks, double denominator_floor,        \
                                           void *stream);                                       \
    /* backward_chunked (full: 8 gradients): persistent_bayes_chunked_d8.cu:632 */               \
    int bssm_d##DN##_backward_chunked(                                                          \
        const float *keys, const float *values, const float *queries, const float *decay,       \
        const float *process, const float *observation, const float *mean0, const float *cov0,  \
        const float *boundary_mean, const float *boundary_cov, const float *grad_out,           \
        const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,            \
        float *grad_values, float *grad_queries, float *grad_decay, float *grad_process,        \
        float *grad_observation, float *grad_mean0, float *grad_cov0, void *workspace,          \
        size_t workspace_bytes, long n, long t, int chunks, double denominator_floor,           \
        void *stream);                                                                          \
    /* backward_chunked_lean (k, v, q gradients): persistent_bayes_chunked_d8.cu:637 */          \
    int bssm_d##DN##_backward_chunked_lean(                                                     \
        const float *keys, const float *values, const float *queries, const float *decay,       \
        const float *process, const float *observation, const float *mean0, const float *cov0,  \
        const float *boundary_mean, const float *boundary_cov, const float *grad_out,           \
        const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,            \
        float *grad_values, float *grad_queries, void *workspace, size_t workspace_bytes,       \
        long n, long t, int chunks, double denominator_floor, void *stream);                    \
    /* backward_chunked_fixed: persistent_bayes_chunked_d8.cu:648 */                             \
    int bssm_d##DN##_backward_chunked_fixed(                                                    \
        const float *keys, const float *values, const float *queries, const float *decay,       \
        const float *process, const float *observation, const float *mean0, const float *cov0,  \
        const float *boundary_mean, const float *boundary_cov, const float *grad_out,           \
        const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,            \
        float *grad_values, float *grad_queries, float *grad_decay, float *grad_process,        \
        float *grad_observation, float *grad_mean0, float *grad_cov0, void *workspace,          \
        size_t workspace_bytes, long n, long t, int chunks, double denominator_floor,           \
        void *stream);                                                                          \
    /* backward_chunked_lean_fixed: persistent_bayes_chunked_d8.cu:642 */                        \
    int bssm_d##DN##_backward_chunked_lean_fixed(                                               \
        const float *keys, const float *values, const float *queries, const float *decay,       \
        const float *process, const float *observation, const float *mean0, const float *cov0,  \
        const float *boundary_mean, const float *boundary_cov, const float *grad_out,           \
        const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,            \
        float *grad_values, float *grad_queries, void *workspace, size_t workspace_bytes,       \
        long n, long t, int chunks, double denominator_floor, void *stream);

BSSM_DECLARE_DIM(1)
BSSM_DECLARE_DIM(2)
BSSM_DECLARE_DIM(4)
BSSM_DECLARE_DIM(8)
BSSM_DECLARE_DIM(64)

/* backward_chunked_noinitial[_fixed] (6 gradients: k, v, q, decay, process,
 * observation): persistent_bayes_chunked_d2m8.cu:576-600. */
int bssm_d2_backward_chunked_noinitial(
    const float *keys, const float *values, const float *queries, const float *decay,
    const float *process, const float *observation, const float *mean0, const float *cov0,
    const float *boundary_mean, const float *boundary_cov, const float *grad_out,
    const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,
    float *grad_values, float *grad_queries, float *grad_decay, float *grad_process,
    float *grad_observation, void *workspace, size_t workspace_bytes, long n, long t,
    int chunks, double denominator_floor, void *stream);
int bssm_d2_backward_chunked_noinitial_fixed(
    const float *keys, const float *values, const float *queries, const float *decay,
    const float *process, const float *observation, const float *mean0, const float *cov0,
    const float *boundary_mean, const float *boundary_cov, const float *grad_out,
    const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,
    float *grad_values, float *grad_queries, float *grad_decay, float *grad_process,
    float *grad_observation, void *workspace, size_t workspace_bytes, long n, long t,
    int chunks, double denominator_floor, void *stream);

/*
 * Allocation-free backward (no counterpart in the reference).
 *
 * For callers that cannot allocate device memory at call time -- a host whose
 * allocator owns the device memory budget, a serving loop that cannot take the
 * device-wide synchronisation an allocation implies, or an FFI host with no
 * device allocator -- this runs the same backward as bssm_backward_chunked_ex
 * (recompute mode: no replay states) with its phase-A scratch in a static
 * device array of bssm_backward_noalloc_max_scratch_bytes() bytes (32 MiB),
 * which every GPU that loads the library holds until the process exits.
 *   - Arguments are those of bssm_backward_chunked_ex without replay_states
 *     and workspace.  Inputs and outputs are still the caller's.
 *   - A problem whose scratch (bssm_backward_workspace_bytes) exceeds the
 *     static size is rejected with BSSM_ERR_WORKSPACE and a message.
 *   - Nothing is allocated or freed (no cudaMalloc / cudaFree).
 *   - The first call on a device looks up the array's device address with
 *     cudaGetSymbolAddress (with that device current) and caches it under the
 *     current CUDA context; make that first call before any stream capture on
 *     that device.  A new context (after a device reset) gets a new lookup.
 *   - All calls on a device share the one array and it keeps the last call's
 *     contents; nothing in it needs to start at zero.  Calls that overlap on
 *     the GPU (concurrent streams, or several host threads on one device)
 *     race on it: serialise them.
 */
size_t bssm_backward_noalloc_max_scratch_bytes(void);
int bssm_backward_chunked_noalloc(int key_dim, int value_dim, int io_dtype, int fixed,
                                  int need_dynamics, int need_initial,
                                  const void *keys, const void *values, const void *queries,
                                  const float *decay, const float *process, const float *observation,
                                  const float *mean0, const float *cov0,
                                  const float *boundary_mean, const float *boundary_cov,
                                  const float *grad_out, const float *grad_mean_final,
                                  const float *grad_cov_final,
                                  void *grad_keys, void *grad_values, void *grad_queries,
                                  float *grad_decay, float *grad_process, float *grad_observation,
                                  float *grad_mean0, float *grad_cov0,
                                  long n, long t, int chunks, double denominator_floor,
                                  void *stream);

/*
 * Rotation dynamics (replaces the dense path of bayes_ssm/bayesian_layer.py:
 * 254-340 for rotation_radii / rotation_angles: the reference has no kernel
 * for it).  Transition A = blockdiag(A_m), A_m = [[c_m, -s_m], [s_m, c_m]]
 * per key pair m, given as cosines[n,t,m] = rho cos(theta) and
 * sines[n,t,m] = rho sin(theta); process noise blockdiag(diag(q_m, 0)) with
 * process[n,t,m] = q_m (>= 0); observation [n,t].  Float32 throughout;
 * (key_dim, value_dim) in {(2,8), (4,8), (8,8)}.  Layouts, boundary states,
 * floor and NULL initial-state conventions as bssm_forward_chunked_ex.  The
 * backward recomputes each chunk into `workspace`
 * (bssm_rotation_workspace_bytes) and writes the gradients of keys, values,
 * queries, cosines, sines, process and observation (and of the initial
 * state when need_initial != 0; the covariance's is symmetric).
 */
/*
 * The rotation coefficients from the caller's radii and angles: cosines[i] =
 * rho_i cos(angles[i]), sines[i] = rho_i sin(angles[i]) with rho the
 * reference's radius handling (bayes_ssm/bayesian_layer.py: rotation_radii
 * clamped below at the smallest normal float and above at 1, then
 * make_rotation_dynamics' exp(log(radius)) clipped at 1), in one pass; the
 * backward gives the radii and angles gradients of that chain (grad_cosines /
 * grad_sines may be NULL for zero).  Float32, `count` elements, contiguous.
 */
int bssm_rotation_coefficients(const float *radii, const float *angles, long count, float *cosines, float *sines,
                               void *stream);
int bssm_rotation_coefficients_backward(const float *radii, const float *angles, const float *grad_cosines,
                                        const float *grad_sines, long count, float *grad_radii, float *grad_angles,
                                        void *stream);
size_t bssm_rotation_workspace_bytes(int key_dim, int value_dim, long n, long t, int chunks);
int bssm_rotation_forward_chunked(int key_dim, int value_dim, const float *keys, const float *values,
                                  const float *queries, const float *cosines, const float *sines,
                                  const float *process, const float *observation, const float *mean0,
                                  const float *cov0, float *out, float *mean_final, float *cov_final,
                                  float *boundary_mean, float *boundary_cov, long n, long t, int chunks,
                                  double denominator_floor, void *stream);
int bssm_rotation_backward_chunked(int key_dim, int value_dim, int need_initial, const float *keys,
                                   const float *values, const float *queries, const float *cosines,
                                   const float *sines, const float *process, const float *observation,
                                   const float *boundary_mean, const float *boundary_cov, const float *grad_out,
                                   const float *grad_mean_final, const float *grad_cov_final, float *grad_keys,
                                   float *grad_values, float *grad_queries, float *grad_cosines,
                                   float *grad_sines, float *grad_process, float *grad_observation,
                                   float *grad_mean0, float *grad_cov0, void *workspace, size_t workspace_bytes,
                                   long n, long t, int chunks, double denominator_floor, void *stream);

/*
 * Input checks of bayesian_layer in one pass (replaces the torch.isfinite(x)
 * .all() and x.min() validation of bayes_ssm/bayesian_layer.py:105-128).
 *
 * Reads n elements of x (BSSM_F32, BSSM_BF16 or BSSM_F16) once on `stream`
 * and ORs into the device word *flags: BSSM_CHECK_NONFINITE if any element
 * is NaN or infinite, BSSM_CHECK_NOT_POSITIVE if any is <= 0,
 * BSSM_CHECK_NEGATIVE if any is < 0.  The caller zeroes *flags first and
 * reads it back (after the stream has run) to raise its own errors.
 */
#define BSSM_CHECK_NONFINITE 1u
#define BSSM_CHECK_NOT_POSITIVE 2u
#define BSSM_CHECK_NEGATIVE 4u
int bssm_check_values(const void *x, long n, int dtype, unsigned *flags, void *stream);

/*
 * BayesianMixer paper-feature prologue (replaces the op chain of
 * example/train_6layer.py:579-700 for the fused Q/K/V + auxiliary projection
 * with learned diagonal dynamics: CausalDepthwise4 :160-191 over the Q/K/V
 * channels, F.silu :629-637, F.normalize of q and k :638-639, softplus noise
 * :665-666, exp(-softplus) decay :698, and the permutes to [B*H, T, .]
 * :647-650,699-701).
 *
 * `projected` is [batch, tokens, row_stride] (BSSM_F32 or BSSM_BF16), whose
 * first 2 SW + W + SW + 2H channels are, in order, the q (SW = heads *
 * key_dim), k (SW) and v (W = heads * head_dim) streams, the decay logits (SW)
 * and the per-head (process, observation) noise pairs (2H).  conv_weight is
 * the Conv1d weight [2 SW + W, 1, 4] as float32; aux_bias [SW + 2H] float32 is
 * added to the auxiliary channels (may be null).  Outputs: keys and queries
 * [batch*heads, tokens, key_dim] and values [batch*heads, tokens, head_dim]
 * in out_dtype; decay [batch*heads, tokens, key_dim], process and observation
 * [batch*heads, tokens] in float32.  key_dim must be a power of two in
 * [2, 64] and head_dim even; row_stride even; tensors 8-byte aligned.
 * check_flags is null or six zeroed words into which the kernel ORs the
 * BSSM_CHECK_* flags of the keys, values, queries, decay, process and
 * observation it writes (in that order), as bssm_check_values would report
 * them -- finiteness only for the first four, all three flags for the noise
 * rows -- so a caller that validates these outputs (bayesian_layer,
 * reference bayesian_layer.py:105-128) need not read them again.
 */
int bssm_envelope_prologue(const void *projected, int in_dtype, long batch, long tokens, int heads, int key_dim,
                           int head_dim, long row_stride, const float *conv_weight, const float *aux_bias,
                           void *keys, void *queries, void *values, int out_dtype, float *decay, float *process,
                           float *observation, unsigned *check_flags, void *stream);

/*
 * Backward of bssm_envelope_prologue.  Gradients of the six outputs (any may
 * be null = zero; keys/queries/values gradients in out_dtype) give
 * grad_projected (the prologue's channels of [batch, tokens,
 * grad_row_stride] in in_dtype; other channels are not written),
 * grad_conv_weight [2 SW + W, 4] and grad_aux_bias [SW + 2H] (null to skip),
 * both float32 and summed deterministically.  `workspace` (32-byte aligned)
 * holds bssm_envelope_partial_floats() floats of per-span partial sums.
 */
long bssm_envelope_partial_floats(long batch, long tokens, int heads, int key_dim, int head_dim);
int bssm_envelope_prologue_backward(const void *projected, int in_dtype, long batch, long tokens, int heads,
                                    int key_dim, int head_dim, long row_stride, const float *conv_weight,
                                    const float *aux_bias, const void *grad_keys, const void *grad_queries,
                                    const void *grad_values, int out_dtype, const float *grad_decay,
                                    const float *grad_process, const float *grad_observation, void *grad_projected,
                                    long grad_row_stride, float *grad_conv_weight, float *grad_aux_bias,
                                    float *workspace, long workspace_floats, void *stream);

/*
 * BayesianMixer readout epilogue (replaces example/train_6layer.py:719-729:
 * the permute of the recurrence's reads to [B, T, H, hd], read.to(x.dtype),
 * nn.RMSNorm(hd) with weight norm_weight and epsilon eps, times SiLU(gate),
 * reshaped to [B, T, W]).  read is [batch*heads, tokens, head_dim]
 * (read_dtype); gate holds rows of at least W = heads * head_dim channels,
 * gate_row_stride elements apart (gate_dtype, which is also the output's
 * dtype and the dtype the reads are rounded to before the norm).  out is
 * [batch, tokens, W].  head_dim is 8, 16, 32 or 64; tensors 16-byte aligned.
 */
int bssm_envelope_epilogue(const void *read, int read_dtype, const void *gate, int gate_dtype, long gate_row_stride,
                           const float *norm_weight, float eps, long batch, long tokens, int heads, int head_dim,
                           void *out, void *stream);
/*
 * Backward of bssm_envelope_epilogue: grad_out [batch, tokens, W] (gate
 * dtype) gives grad_read (read layout and dtype), grad_gate (rows
 * grad_gate_row_stride apart, gate dtype) and grad_norm_weight [head_dim]
 * (float32, summed in a fixed order).  workspace holds
 * bssm_envelope_epilogue_partial_floats() floats.
 */
long bssm_envelope_epilogue_partial_floats(long batch, long tokens, int heads, int head_dim);

/*
 * nn.RMSNorm over rows of `width` elements (the mixer's input norm,
 * example/train_6layer.py:581): out = x * rsqrt(mean(x^2) + eps) * weight,
 * computed in float32, stored in x's dtype (BSSM_F32 or BSSM_BF16).  width is
 * 256, 512, 768 or 1024; x and out [rows, width] contiguous; weight float32.
 * The backward writes grad_x (x's dtype) and grad_weight (float32, summed in
 * a fixed order; workspace of bssm_rms_norm_partial_floats() floats).
 */
int bssm_rms_norm(const void *x, int dtype, long rows, int width, const float *weight, float eps, void *out,
                  void *stream);
long bssm_rms_norm_partial_floats(long rows, int width);
int bssm_rms_norm_backward(const void *x, int dtype, long rows, int width, const float *weight, float eps,
                           const void *grad_out, void *grad_x, float *grad_weight, float *workspace,
                           long workspace_floats, void *stream);
int bssm_envelope_epilogue_backward(const void *read, int read_dtype, const void *gate, int gate_dtype,
                                    long gate_row_stride, const float *norm_weight, float eps, long batch, long tokens,
                                    int heads, int head_dim, const void *grad_out, void *grad_read, void *grad_gate,
                                    long grad_gate_row_stride, float *grad_norm_weight, float *workspace,
                                    long workspace_floats, void *stream);

/*
 * Device status (no counterpart in the reference: its kernels have no waits).
 *
 * The thread-per-chain kernels wait on shared-memory barriers for their own
 * asynchronous copies.  Every such wait is bounded: one that gives up is
 * counted in a device word and the kernel runs on (its outputs are then
 * wrong) instead of hanging the GPU.  bssm_stream_status synchronises
 * `stream` and returns BSSM_ERR_TIMEOUT, with a message, when the current
 * device's count has grown since the previous bssm_stream_status call on
 * that device (each give-up is reported once), BSSM_ERR_CUDA for a CUDA
 * error, else BSSM_OK.  The word is device-wide: a give-up on another stream
 * of the same device is reported too.  The Python layer calls this after
 * every forward and backward launch (outside CUDA graph capture) and raises.
 */
int bssm_stream_status(void *stream);

/*
 * Diagnostics (no counterpart in the reference).
 *
 * bssm_debug_wait_timeouts: the give-up count on the current device since
 * the library was loaded -- 0 in a healthy process.  It synchronises the
 * device.
 * bssm_debug_wait_probe: launches one thread that waits, polling `limit`
 * times (1..65536), on a barrier phase nothing completes, so its bounded wait
 * gives up and is counted like a give-up inside a recurrence kernel; it
 * tests the reporting path without faulting or hanging anything.
 */
unsigned int bssm_debug_wait_timeouts(void);
int bssm_debug_wait_probe(int limit, void *stream);

/*
 * FP32 FMA throughput probe (measurement only): `blocks` CTAs of 256 threads,
 * each running 8 independent FMA chains for 8 * iters steps, enqueued on
 * `stream`; bssm_debug_fma_probe_flops gives its flop count (FMA = 2), so
 * flops / CUDA-event time is the GPU's achievable FP32 (non-tensor) rate at
 * its current clocks.  out holds blocks * 256 floats; it is not written.
 */
int bssm_debug_fma_probe(float *out, int blocks, int iters, void *stream);
long bssm_debug_fma_probe_flops(int blocks, int iters);

/*
 * Kernel family that served the calling thread's last forward or backward
 * call: 1 thread-per-chain, 2 staged, 3 per-lane, 4 the (64,64) tile
 * kernels; 0 before any call.  The
 * library picks by shape and batch size; the environment variable
 * BSSM_KERNELS=chain|staged|v1, read at every call, forces a family where it
 * supports the shape.
 */
int bssm_debug_last_family(void);

#ifdef __cplusplus
}
#endif

#endif /* BAYES_SSM_B200_H */

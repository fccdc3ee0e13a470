/*
 * sparc_b200.h -- C ABI of the B200-native SPARC hot path (libsparc_b200.so).
 *
 * Plain pointers and sizes only. Every tensor pointer is a CUDA device pointer to a dense,
 * row-major (last dimension fastest) array. Activations are float32 or bfloat16 (`dtype`);
 * parameters, recurrent states and parameter gradients are float32. `stream` is a
 * cudaStream_t passed as void*. All entry points only enqueue work on that stream (no host
 * synchronisation) except sparc_read_status.
 *
 * Return value: SPARC_OK (0) or a negative SPARC_ERR_* code; sparc_last_error() then returns a
 * message (thread-local). No entry point allocates memory: scratch comes from a caller-owned
 * workspace whose size the *_workspace_bytes query returns. A workspace must be zero-filled
 * once when it is allocated, and may then be reused by any number of launches that are
 * ordered on one stream; calls that run concurrently need distinct workspaces.
 *
 * The mixer runs as chunk summaries -> a carry scan (one thread-block cluster per row, spans of
 * chunks composed in a fixed order) -> a replay; every result, parameter gradients included,
 * is bitwise reproducible run to run. The real-mode scan passes its carries by decoupled
 * lookback (a tile composes whatever predecessor aggregates are ready). Every wait is bounded
 * by `max_spin` polls (0 selects the default, about a second): the lookback's and the TMA
 * copies'; a wait that runs out sets the SPARC_STATUS_TIMEOUT bit in the workspace's status
 * word, continues (with a zero carry in the lookback), and the launch still completes.
 * sparc_read_status reads that word.
 *
 * Which reference interface each entry point replaces (paths inside Botwwt/sparc):
 *   sparc_mixer_forward   SPARCMixer.forward -> run_sequence          sparc-kernal/sparc.py:90-91,
 *                         forward/scan.py:1398-1603 (make_controls forward/control.py:129-139,
 *                         latest_sparc_write backward/control.py:92-111,
 *                         _SPARCChunkScan.forward backward/scan.py:1126-1372, cat+relu
 *                         forward/scan.py:1598-1603; with return_cache the last state as in
 *                         sparc_scan_with_last backward/scan.py:1857-1877; h0 as in
 *                         _SPARCTiledSerialScan backward/scan.py:971-1070)
 *   sparc_mixer_backward  autograd backward of the above: _SPARCChunkScan.backward
 *                         backward/scan.py:1375-1640, _LatestSPARCWrite.backward
 *                         backward/control.py:113-129, torch autograd of make_controls;
 *                         grad of h0 / of the returned last state as in
 *                         _SPARCTiledSerialScan.backward backward/scan.py:1034-1070
 *   sparc_decode_step     SPARCMixer.step -> run_decode_step -> latest_sparc_decode
 *                         sparc.py:122-123, forward/decode.py:273-306, 58-75 (kernel 11-55)
 *   sparc_real_scan_forward   real_scan / real_chunk_scan / real_scan_with_last forward
 *                         backward/scan.py:793-855, 1643-1650, 1821-1834
 *   sparc_real_scan_backward  _RealScan.backward / _RealChunkScan.backward
 *                         backward/scan.py:811-822, 857-884
 */
#ifndef SPARC_B200_H_
#define SPARC_B200_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SPARC_OK 0
#define SPARC_ERR_ARG (-1)       /* null or inconsistent pointer arguments */
#define SPARC_ERR_SHAPE (-2)     /* unsupported or invalid shape */
#define SPARC_ERR_DTYPE (-3)     /* unsupported activation dtype */
#define SPARC_ERR_WORKSPACE (-4) /* workspace missing or smaller than the query returned */
#define SPARC_ERR_LAUNCH (-5)    /* CUDA launch / runtime error */

#define SPARC_DTYPE_F32 0
#define SPARC_DTYPE_BF16 1

#define SPARC_STATUS_TIMEOUT 1u  /* a lookback wait ran out of polls */

/* Forward of one SPARC mixer layer: y = relu([Re h, Im h]) for the recurrence
 * h_t = a_t h_{t-1} + b_t over M = width/2 complex modes, with a_t, b_t computed from x_t
 * and the parameters. `carry` receives the state at the end of every chunk of
 * sparc_mixer_chunk_tokens(dtype) tokens ([batch, sparc_mixer_carry_chunks(length, dtype), M] complex,
 * interleaved real/imag float32) and `controls` the per-token controls ([batch, length,
 * sparc_mixer_controls_floats()] float32: e^eta, delta, tanh p0, tanh p1, keep (0 at a reset
 * token), the block's norm scale and the raw projections, laid out as pairs for the kernels);
 * the backward needs both, and y. h0 (initial state) and last (final
 * state) are optional pairs (NULL, NULL). `reset` (optional, [batch, length] bytes) marks the
 * tokens where a new segment starts: there the transition is zero, so the state restarts from
 * the token's write, as with segment_pos == 0 (or reset_first at t = 0) in the reference's
 * tiled serial scan (forward/scan.py:807-854, common.py:219-268). */
/* Block mode (norm_weight given): one layer of the config-5 stack, out = x + relu([Re h, Im h])
 * where the mixer runs on n = RMSNorm(x) = x * r * norm_weight, r = (mean(x^2) + norm_eps)^(-1/2)
 * per token, computed inside the mixer kernels (no separate norm or residual pass); y receives
 * `out`, and relu_mask the bits of relu(h) > 0 that the backward needs in place of y. The
 * backward then returns the block input's gradient in dx (the residual path included) and the
 * norm weight's in grad_norm_weight. */
/* Projection mode (projections given): the recurrence core of the projection variant, the JAX
 * sequence layer and RTRL cell of sparc-impl (recurrence.py:20-63, layers.py:88-126), whose
 * content and controls come from matrix products the caller computes: x is the content input
 * u = [x_in content_real, x_in content_imag] ([batch, length, width], width = 2M), projections
 * the per-token controller projections p = [x_in, 1] phase_controller / retention_controller
 * ([batch, length, 2] float32, bias included), and y receives the states [Re h, Im h] with no
 * relu (the caller's readout follows). The content is tanh(u), or u with content_linear
 * (content_activation "linear"). The directions are not read (may be NULL). The backward takes
 * dy on the states and returns the content input's gradient in dx and the projections' in
 * grad_projections; the caller finishes x_in's and the matrices' gradients with the transposed
 * products. */
/* Scan-level mode (projections given and content_linear == 2): the reference's scan-level
 * functions (sparc_scan, sparc_chunk_scan, sparc_tiled_serial_scan, sparc_scan_with_last,
 * sparc_training_scan_dispatch; backward/scan.py:922-1070, 1124-1372, 1658-1877, math at
 * forward/scan.py:725-757), whose per-token controls and writes are given: projections holds
 * (delta, eta) per token ([batch, length, 2] float32, any values), x the writes
 * [b_r, b_i] ([batch, length, width]), and the recurrence is h_t = rho e^{i phi} h_{t-1} + b_t
 * with rho = exp(-e^{nu_log} e^eta), phi = e^{theta_log} + (1 - rho) delta (no write gain; the
 * write parameters are not read and their gradients come back zero). y receives the states
 * [Re h, Im h] with no relu, or, with y_im given, Re h in y and Im h in y_im (each
 * [batch, length, M]). The backward returns the writes' gradient in dx and (d delta, d eta)
 * per token in grad_projections. */
typedef struct SparcMixerFwdArgs {
  const void* x;                       /* [batch, length, width]  activations (dtype) */
  void* y;                             /* [batch, length, width]  output (dtype) */
  const float* nu_log;                 /* [M] */
  const float* theta_log;              /* [M] */
  const float* phase_direction;        /* [width + 1] (last entry is the bias) */
  const float* radial_direction;       /* [width + 1] */
  const float* write_log_gain;         /* [M] */
  const float* write_phase_response;   /* [M] */
  const float* write_radial_response;  /* [M] */
  const float* h0_r;                   /* [batch, M] or NULL */
  const float* h0_i;                   /* [batch, M] or NULL */
  float* last_r;                       /* [batch, M] or NULL */
  float* last_i;                       /* [batch, M] or NULL */
  float* carry;                        /* [batch, chunks, M, 2] */
  float* controls;                     /* [batch, length, sparc_mixer_controls_floats()] */
  const unsigned char* reset;          /* [batch, length] (nonzero = segment start) or NULL */
  const float* norm_weight;            /* [width]: the call is a block (below), or NULL */
  float norm_eps;                      /* block: RMSNorm epsilon */
  unsigned* relu_mask;                 /* block: [batch, length, sparc_mixer_mask_words(width)] out */
  const float* projections;            /* [batch, length, 2]: projection mode (above), or NULL */
  int content_linear;                  /* projection mode: 1 = content u instead of tanh(u);
                                          2 = the scan-level mode (above) */
  void* workspace;
  size_t workspace_bytes;
  long long batch;
  long long length;
  int width;
  int dtype;                           /* SPARC_DTYPE_* */
  unsigned max_spin;                   /* bound of the TMA waits (0 = default) */
  void* y_im;                          /* scan-level mode: Im h [batch, length, M] out (y then
                                          holds Re h [batch, length, M]), or NULL */
  void* states;                        /* [batch, length, width] out (dtype): every token's state,
                                          Re h in columns [0, M), Im h in [M, width) (the layout of
                                          y), for the backward's `states`; or NULL. Plain and block
                                          mode only (the other modes' y holds the states). Costs
                                          one activation-sized write here and saves the backward
                                          its replay of the states (the reference's backward
                                          likewise reads saved states, backward/scan.py:1375-1640) */
} SparcMixerFwdArgs;

/* Backward of sparc_mixer_forward for the loss gradient dy on y (and optionally grad_last on
 * the returned last state). Writes dx and every parameter gradient (energy_response's is 0:
 * the reference multiplies that parameter by zero). Parameter gradients are reduced in a
 * fixed order (deterministic run to run). */
typedef struct SparcMixerBwdArgs {
  const void* x;                       /* [batch, length, width] forward input (dtype) */
  const void* y;                       /* [batch, length, width] the forward's output (dtype);
                                          not read by a block or in projection mode */
  const void* dy;                      /* [batch, length, width] (dtype) */
  void* dx;                            /* [batch, length, width] (dtype) */
  const float* nu_log;
  const float* theta_log;
  const float* phase_direction;
  const float* radial_direction;
  const float* write_log_gain;
  const float* write_phase_response;
  const float* write_radial_response;
  const float* h0_r;                   /* as given to the forward, or NULL */
  const float* h0_i;
  const float* grad_last_r;            /* [batch, M] or NULL */
  const float* grad_last_i;
  float* grad_h0_r;                    /* [batch, M] or NULL */
  float* grad_h0_i;
  const float* carry;                  /* the forward's carry output */
  const float* controls;               /* the forward's controls output */
  const float* norm_weight;            /* block: as given to the forward, else NULL */
  const unsigned* relu_mask;           /* block: the forward's relu_mask output */
  float* grad_norm_weight;             /* block: [width] */
  float* grad_nu_log;                  /* [M] */
  float* grad_theta_log;               /* [M] */
  float* grad_phase_direction;         /* [width + 1] (NULL in projection mode) */
  float* grad_radial_direction;        /* [width + 1] (NULL in projection mode) */
  float* grad_write_log_gain;          /* [M] */
  float* grad_energy_response;         /* [M], written with zeros */
  float* grad_write_phase_response;    /* [M] */
  float* grad_write_radial_response;   /* [M] */
  float* grad_projections;             /* projection mode: [batch, length, 2] out, else NULL */
  int content_linear;                  /* projection / scan-level mode: as given to the forward */
  void* exchange_buffers[8];           /* data parallelism: every rank's exchange buffer (below) */
  int exchange_world;                  /* > 1: the parameter gradients are summed over the ranks */
  int exchange_rank;
  unsigned* exchange_status;           /* device word, or'ed with 16 if an exchange wait ran out */
  void* workspace;
  size_t workspace_bytes;
  long long batch;
  long long length;
  int width;
  int dtype;
  unsigned max_spin;
  const void* states;                  /* the forward's `states` output (in projection mode: its
                                          output y), or NULL. With it (and 16-byte aligned rows:
                                          the condition of the tensor maps) the gradient kernel
                                          reads the states instead of replaying them from the
                                          chunk carries; its sign stands in for y's relu mask,
                                          so y may then be NULL. Not used in the scan-level mode */
} SparcMixerBwdArgs;

/* Fused cross-GPU gradient sum (batch-sharded data parallelism, up to 8 ranks of one node):
 * with exchange_world > 1 the backward's parameter-gradient reduction kernel also sums every
 * gradient over the ranks through NVLink peer memory before writing it, so the gradients it
 * returns are already the group's sums (no separate all-reduce). Each rank allocates one buffer
 * of sparc_exchange_buffer_bytes(world) bytes with sparc_peer_buffer_alloc (zeroed, with its
 * IPC handle), the handles are exchanged by the caller and opened with sparc_peer_buffer_open;
 * exchange_buffers[r] is rank r's buffer as mapped in this process. Every rank must make the
 * same sequence of backward calls with the same shapes. */
size_t sparc_exchange_buffer_bytes(int world);

/* One fused decode step (forward/decode.py:11-55): x [batch, width] (dtype), state
 * [batch, M] float32 in; y [batch, width] (dtype), new state [batch, M] float32 out. The new
 * state may not alias the old one. */
typedef struct SparcDecodeArgs {
  const void* x;
  void* y;
  const float* state_r;
  const float* state_i;
  float* new_state_r;
  float* new_state_i;
  const float* nu_log;
  const float* theta_log;
  const float* phase_direction;
  const float* radial_direction;
  const float* write_log_gain;
  const float* write_phase_response;
  const float* write_radial_response;
  long long batch;
  int width;
  int dtype;
} SparcDecodeArgs;

/* Real diagonal scan h_t = a_t h_{t-1} + b_t over [batch, length, channels]
 * (backward/scan.py:793-884, 1643-1650, 1821-1834; kernels forward/scan.py:622-698,
 * backward/scan.py:35-128). As in the reference, a is read in its own dtype `a_dtype` and
 * widened to float32, b and out are in `dtype` (b's), and the recurrence and its carries are
 * float32; the backward writes grad_a in a_dtype and reads grad_out / writes grad_b in dtype.
 * `carry` ([batch, sparc_real_carry_chunks(length), channels] float32) receives the state at
 * the end of each chunk for the backward; `last` ([batch, channels] float32) is optional. */
typedef struct SparcRealFwdArgs {
  const void* a;
  const void* b;
  void* out;
  float* last;                         /* or NULL */
  float* carry;
  void* workspace;
  size_t workspace_bytes;
  long long batch;
  long long length;
  long long channels;
  int dtype;                           /* b and out */
  int a_dtype;                         /* a */
  unsigned max_spin;
  int inject_enable;                   /* test hook: 1 = tile inject_tile never publishes */
  long long inject_tile;               /*   (its successor's bounded wait runs out) */
} SparcRealFwdArgs;

typedef struct SparcRealBwdArgs {
  const void* a;
  const void* b;
  const void* grad_out;
  const float* carry;                  /* the forward's carry output */
  void* grad_a;
  void* grad_b;
  void* workspace;
  size_t workspace_bytes;
  long long batch;
  long long length;
  long long channels;
  int dtype;                           /* b, grad_out and grad_b */
  int a_dtype;                         /* a and grad_a */
  unsigned max_spin;
} SparcRealBwdArgs;

const char* sparc_last_error(void);

long long sparc_mixer_chunk_tokens(int dtype);
long long sparc_mixer_carry_chunks(long long length, int dtype);
/* Floats per token of the forward's controls output (16). */
int sparc_mixer_controls_floats(void);
/* 32-bit words per token of a block's relu_mask (four per 64 modes, whole CTAs of 256 modes). */
int sparc_mixer_mask_words(int width);
size_t sparc_mixer_workspace_bytes(long long batch, long long length, int width, int dtype);
int sparc_mixer_forward(const SparcMixerFwdArgs* args, void* stream);
int sparc_mixer_backward(const SparcMixerBwdArgs* args, void* stream);

/* No counterpart in the reference: an extra entry point of this library.
 * sparc_mixer_forward_noalloc runs exactly the computation of sparc_mixer_forward but takes
 * no workspace (args->workspace and args->workspace_bytes are ignored). It is for callers
 * that cannot allocate device memory: for example a plugin bound through an FFI into a host
 * process whose own memory pool has already claimed the GPU, or a serving loop that must not
 * call cudaMalloc after start-up because it can block the whole device. Its scratch is a
 * fixed array of sparc_mixer_noalloc_scratch_bytes() (32 MiB) inside the library. The array
 * belongs to the library's mixer module, so every GPU on which any mixer kernel of this
 * library runs (through this entry point or any other) holds it until the process exits.
 * A problem whose forward scratch, sparc_mixer_noalloc_scratch_needed(batch, length, width,
 * dtype) bytes (a 256-byte header plus 16 bytes per (batch row, chunk of C tokens, mode) with
 * the modes rounded up to whole 256-mode tiles; C = 16 for bfloat16, 8 for float32), is
 * larger is rejected with SPARC_ERR_WORKSPACE and a message. The first call on a device looks
 * up that device's copy of the array (cudaGetSymbolAddress), so make it before any stream
 * capture. All calls share the array: calls whose executions overlap on the GPU (other
 * streams, other host threads) race and must be serialised by the caller. The caller still
 * provides x, y, carry, controls and the parameters.
 * The array's status word (SPARC_STATUS_* bits; a timed-out wait of a tile kernel sets
 * SPARC_STATUS_TIMEOUT) is sticky: it stays set for every later call on that device until
 * sparc_mixer_noalloc_clear_status clears it. sparc_mixer_noalloc_read_status reads it (and
 * synchronises `stream`); neither allocates. */
size_t sparc_mixer_noalloc_scratch_bytes(void);
size_t sparc_mixer_noalloc_scratch_needed(long long batch, long long length, int width, int dtype);
int sparc_mixer_forward_noalloc(const SparcMixerFwdArgs* args, void* stream);
int sparc_mixer_noalloc_read_status(unsigned* status, void* stream);
int sparc_mixer_noalloc_clear_status(void* stream);

int sparc_decode_step(const SparcDecodeArgs* args, void* stream);

/* Tokens per saved carry of the real-mode scan (32); sparc_real_carry_chunks(length) is
 * ceil(length / sparc_real_chunk_tokens()). */
long long sparc_real_chunk_tokens(void);
long long sparc_real_carry_chunks(long long length);
size_t sparc_real_workspace_bytes(long long batch, long long length, long long channels, int dtype);
int sparc_real_scan_forward(const SparcRealFwdArgs* args, void* stream);
int sparc_real_scan_backward(const SparcRealBwdArgs* args, void* stream);

/* Generic complex diagonal scan h_t = a_t h_{t-1} + b_t (h_{-1} = 0) over [batch, length,
 * modes], each part a separate contiguous array (backward/scan.py:887-919, 1653-1656, 1838-1855;
 * kernels forward/scan.py:701-722, backward/scan.py:131-160). ar, ai are read in a_dtype and br,
 * bi in b_dtype, widened to float32; out_r, out_i are written in b_dtype; last_r, last_i
 * ([batch, modes] float32, optional) receive the final state. The backward reads the forward's
 * outputs (b_dtype) as the previous states and grad_out_r/_i in b_dtype, and writes grad_ar,
 * grad_ai, grad_br, grad_bi in a_dtype (grad_ar = Re(adj) Re(h_{t-1}) + Im(adj) Im(h_{t-1}),
 * grad_ai = Im(adj) Re(h_{t-1}) - Re(adj) Im(h_{t-1}), grad_b = adj, with
 * adj_t = grad_t + conj(a_{t+1}) adj_{t+1}). `workspace`: sparc_complex_workspace_bytes bytes,
 * 16-byte aligned, no initial contents needed. Shapes: batch <= 65535, ceil(length / 32) <=
 * 65535, batch x ceil(length / 32) x modes < 2^31. */
typedef struct SparcComplexFwdArgs {
  const void* ar;
  const void* ai;
  const void* br;
  const void* bi;
  void* out_r;
  void* out_i;
  float* last_r;                       /* or NULL (with last_i) */
  float* last_i;
  void* workspace;
  size_t workspace_bytes;
  long long batch;
  long long length;
  long long modes;
  int a_dtype;
  int b_dtype;
} SparcComplexFwdArgs;

typedef struct SparcComplexBwdArgs {
  const void* ar;
  const void* ai;
  const void* out_r;                   /* the forward's outputs */
  const void* out_i;
  const void* grad_out_r;
  const void* grad_out_i;
  void* grad_ar;
  void* grad_ai;
  void* grad_br;
  void* grad_bi;
  void* workspace;
  size_t workspace_bytes;
  long long batch;
  long long length;
  long long modes;
  int a_dtype;
  int b_dtype;
} SparcComplexBwdArgs;

long long sparc_complex_chunk_tokens(void);
size_t sparc_complex_workspace_bytes(long long batch, long long length, long long modes);
int sparc_complex_scan_forward(const SparcComplexFwdArgs* args, void* stream);
int sparc_complex_scan_backward(const SparcComplexBwdArgs* args, void* stream);

/* Diagnostics: per-kernel device time. While enabled, every kernel launch of this library is
 * bracketed by CUDA events on its stream (launches inside a stream capture are not timed).
 * sparc_timing_read waits for the recorded launches, writes per-kernel totals (milliseconds) and
 * launch counts for up to n kernel kinds (either pointer may be NULL), resets them, and returns
 * the number of kernel kinds, SPARC_TIMING_KERNELS; sparc_timing_kernel_name names kind `id`.
 * sparc_timing_enable returns the previous setting. */
#define SPARC_TIMING_KERNELS 23
int sparc_timing_enable(int on);
const char* sparc_timing_kernel_name(int id);
int sparc_timing_read(double* ms, long long* launches, int n);

/* Status word of a workspace (SPARC_STATUS_* bits). Reads synchronise `stream`. */
int sparc_read_status(const void* workspace, unsigned* status, void* stream);
int sparc_clear_status(void* workspace, void* stream);

/* RTRL online traces of the SPARC cell (sparc-impl/sparc/training/rtrl.py:61-148, replaces the
 * JAX _trace_step / stored_rtrl_step). Traces and states are complex, stored as interleaved
 * float32 pairs (the layout of complex64): trace index 0-4 the modal parameters decay_log,
 * frequency_log, write_log_gain, write_phase_response, write_retention_response [batch, M];
 * 5, 6 content_real, content_imag [batch, input_size, M]; 7, 8 phase_controller,
 * retention_controller [batch, input_size + 1, M]. `content` is the caller's product
 * [x content_real, x content_imag] ([batch, 2M] float32) and `projections` [x, 1] phase_controller,
 * [x, 1] retention_controller ([batch, 2] float32). Where reset[b] is nonzero the carried state
 * and traces of row b are zeroed before the step (_reset_carry, rtrl.py:49-58). new_traces may
 * alias traces (each element is read and written by the same thread). `saved`
 * ([batch, M, sparc_rtrl_saved_floats()] float32) receives what sparc_rtrl_grad needs. */
typedef struct SparcRtrlStepArgs {
  const float* x;                      /* [batch, input_size] */
  const float* content;                /* [batch, 2M] */
  const float* projections;            /* [batch, 2] */
  const unsigned char* reset;          /* [batch] or NULL */
  const float* state;                  /* [batch, M] complex */
  float* new_state;                    /* [batch, M] complex out */
  const float* decay_log;              /* [M] */
  const float* frequency_log;          /* [M] */
  const float* write_log_gain;         /* [M] */
  const float* write_phase_response;   /* [M] */
  const float* write_retention_response; /* [M] */
  const float* traces[9];
  float* new_traces[9];
  float* saved;
  long long batch;                     /* at most 65535 */
  int input_size;
  int modes;
  int content_linear;                  /* content_activation "linear": content u, else tanh(u) */
} SparcRtrlStepArgs;

/* Gradients of a loss on the step's new state (stored_rtrl_step's backward, rtrl.py:127-148):
 * grad_state holds (dL/dRe h', dL/dIm h') per mode; every parameter's gradient is
 * sum_b (dL/dRe h' Re(trace) + dL/dIm h' Im(trace)) over the step's NEW traces (summed over the
 * modes too for the controllers; grad_params in the trace order, shapes [M], [input_size, M],
 * [input_size + 1]); grad_content [batch, 2M] and grad_projections [batch, 2] are the one-step
 * gradients of the step's content and projection inputs (the caller's products finish the
 * input's). Sums run in a fixed order. */
typedef struct SparcRtrlGradArgs {
  const float* grad_state;             /* [batch, M] complex */
  const float* traces[9];              /* the step's new traces */
  const float* saved;                  /* the step's saved output */
  float* grad_params[9];
  float* grad_content;                 /* [batch, 2M] out */
  float* grad_projections;             /* [batch, 2] out */
  long long batch;
  int input_size;
  int modes;
} SparcRtrlGradArgs;

int sparc_rtrl_saved_floats(void);
int sparc_rtrl_step(const SparcRtrlStepArgs* args, void* stream);
int sparc_rtrl_grad(const SparcRtrlGradArgs* args, void* stream);
const char* sparc_rtrl_last_error(void);

/* Tensor-core product of the projection variant (content, readout and their adjoints; the JAX
 * layer's x @ content_real/imag and states @ readout^T, recurrence.py:39-40, layers.py:125-126):
 *   out[m, n] = sum_k a[m, k] b[n, k] (+ skip[n] x[m, n]) (+ dp[m, 0] c0[n] + dp[m, 1] c1[n])
 * a [rows, k] and b [n, k] row-major bfloat16 (k a multiple of 8, 16-byte aligned bases),
 * float32 accumulation, out [rows, n] bfloat16 (or float32 with out_f32). x (bfloat16,
 * [rows, n]) with skip ([n] float32), and dp ([rows, 2] float32) with c0, c1 ([n] float32),
 * are optional fused terms. `status` (device word) is or'ed with 4 if a bounded wait ran out.
 * With a_mn (b_mn) the operand is stored transposed, a as [k, rows] (b as [k, n]), with rows
 * (n) a multiple of 8 instead of k: the weight gradients x^T du and dy^T h, which contract over
 * the tokens, run on x [tokens, width] and du [tokens, 2M] as they are (no transposed copies).
 * Products with fewer output tiles (128 x 256) than SMs and a long k (the weight gradients of
 * narrow layers) are split along k when `workspace` holds sparc_proj_gemm_workspace_bytes(rows,
 * n, k) bytes (16-byte aligned; 0 bytes needed means no split): each k range's partial product
 * is written there and a second launch adds them in order with the fused terms. A null or
 * smaller workspace gives the unsplit product (same value to rounding).
 *
 * Column sums of the layer's backward (the controller projections' and the skip's gradients,
 * layers.py:112-126): for x [rows, w] (dtype), dp [rows, 2] float32 and, optionally, dy
 * [rows, w] (dtype), sparc_proj_colsum writes d_ctl [w + 1, 2] float32 (column j < w:
 * sum_r x[r, j] dp[r, :], row w: sum_r dp[r, :]) and, with dy, d_skip [w] float32
 * (sum_r dy[r, j] x[r, j]), in a fixed order (bitwise reproducible). `workspace` holds the
 * partial sums: sparc_proj_colsum_workspace_bytes(rows, w) bytes. */
typedef struct SparcProjColsumArgs {
  const void* x;
  const float* dp;
  const void* dy;                      /* or NULL (no d_skip) */
  float* d_ctl;
  float* d_skip;                       /* or NULL */
  void* workspace;
  size_t workspace_bytes;
  long long rows;
  int w;
  int dtype;
} SparcProjColsumArgs;
size_t sparc_proj_colsum_workspace_bytes(long long rows, int w);
int sparc_proj_colsum(const SparcProjColsumArgs* args, void* stream);

/* The layer forward's controller projections (layers.py:112-117, recurrence.py:20-38):
 * p[r, :] = sum_j x[r, j] c[j, :] + c[w, :] for x [rows, w] (dtype) and c [w + 1, 2] float32
 * (phase and retention controllers side by side, the biases in row w); p [rows, 2] float32. */
typedef struct SparcProjRowdotArgs {
  const void* x;
  const float* c;
  float* p;
  long long rows;
  int w;
  int dtype;
} SparcProjRowdotArgs;
int sparc_proj_rowdot(const SparcProjRowdotArgs* args, void* stream);

typedef struct SparcProjGemmArgs {
  const void* a;
  const void* b;
  void* out;
  const void* x;
  const float* skip;
  const float* dp;
  const float* c0;
  const float* c1;
  unsigned* status;
  long long rows;
  int n;
  int k;
  int out_f32;
  unsigned max_spin;                   /* bound of the mbarrier waits (0 = default) */
  int a_mn;                            /* 1: a is stored transposed, [k, rows] (M-major) */
  int b_mn;                            /* 1: b is stored transposed, [k, n] (N-major) */
  void* workspace;                     /* split-k partials, or NULL */
  size_t workspace_bytes;
} SparcProjGemmArgs;

size_t sparc_proj_gemm_workspace_bytes(long long rows, int n, int k);
int sparc_proj_gemm(const SparcProjGemmArgs* args, void* stream);
const char* sparc_proj_gemm_last_error(void);

/* Parameter-gradient all-reduce over NVLink peer memory (batch-sharded data parallelism: the
 * one exchange step; replaces the NCCL all-reduce of the concatenated gradients). Each rank
 * allocates one buffer of sparc_peer_buffer_bytes(world, total) bytes (sparc_peer_buffer_alloc,
 * zeroed, with its CUDA IPC handle), the handles are exchanged by the caller (any host
 * collective), and each rank opens the others' (sparc_peer_buffer_open). sparc_peer_allreduce
 * then sums the float32 gradient segments (in order, `total` floats) over the ranks in place:
 * every rank gets the identical sum in rank order, times `scale`. One kernel: each CTA pushes
 * its slice into every rank's buffer, every value stored with the launch's epoch as one 8-byte
 * word, and waits (bounded by max_spin polls; a wait that runs out or's 8 into *status) until
 * its words from every rank carry the epoch. Every rank must call it the same number of times
 * with the same total. inject_skip_publish (tests only) withholds this rank's push so that the
 * peers' waits run out. */
#define SPARC_PEER_MAX_RANKS 8
#define SPARC_PEER_MAX_SEGMENTS 64
typedef struct SparcPeerAllreduceArgs {
  float* segments[SPARC_PEER_MAX_SEGMENTS];
  long long counts[SPARC_PEER_MAX_SEGMENTS];
  int nseg;
  long long total;
  void* buffers[SPARC_PEER_MAX_RANKS]; /* every rank's buffer as mapped in this process (own included) */
  int world;
  int rank;
  float scale;
  unsigned max_spin;
  unsigned* status;
  int inject_skip_publish;
} SparcPeerAllreduceArgs;

size_t sparc_peer_buffer_bytes(int world, long long total);
int sparc_peer_buffer_alloc(size_t bytes, void** ptr, void* ipc_handle /* 64 bytes out */);
int sparc_peer_buffer_open(const void* ipc_handle, void** ptr);
int sparc_peer_buffer_close(void* ptr);
int sparc_peer_buffer_free(void* ptr);
int sparc_peer_allreduce(const SparcPeerAllreduceArgs* args, void* stream);
const char* sparc_peer_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* SPARC_B200_H_ */

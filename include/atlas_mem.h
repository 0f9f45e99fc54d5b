/*
 * atlas_mem.h -- C ABI of the B200 memory-update library (libatlas_mem.so).
 *
 * The library computes the Titans-RNN / OmegaNet-RNN memory recurrence of
 * atlas_pytorch/rnn_memory.py for N = batch*heads independent units:
 *
 *   phi_t = fmap(k_t), psi_t = fmap(q_t)                     rnn_memory.py:637-642
 *   delta_t = S_ref phi_t - v_t                                rnn_memory.py:659-660
 *   g_t = sum_{j<e} W(t, t-j) delta_{t-j} phi_{t-j}^T          rnn_memory.py:663-687
 *   Z_t = beta_t Z_{t-1} + g_t                                 rnn_memory.py:698
 *   S_t = alpha_t S_{t-1} - eta_t Z_t                          rnn_memory.py:699-700
 *   y_t = S_{t-1} psi_t                                        rnn_memory.py:712-717
 *   S_end = clamp(S_T, -100, 100), Z_end = Z_T                 rnn_memory.py:701-702
 *   buf_out = last e-1 window terms                            rnn_memory.py:684
 *
 * with forward and backward. It replaces the reference's kernel-level entry
 * AtlasOmegaFunction.apply(phi_k, phi_q, v, S_ref, lr, decay, beta, gate, S0, Z0)
 * (atlas_pytorch/cuda/atlas_omega_autograd.py:98-153) and its pybind entries
 * forward_exact / backward_exact (atlas_pytorch/cuda/atlas_omega.cpp:139-142),
 * generalised to every window e, head size, feature map and momentum setting,
 * and with the PyTorch path's semantics (clamped S_end, carried omega buffer).
 *
 * Conventions
 *  - Every pointer is a device pointer to a dense row-major (contiguous) array.
 *  - Token-major tensors are [N, T, dim]; per-token scalars are [N, T];
 *    window gates are [N, T, e]; states are [N, d_v, d_phi]; the omega buffer
 *    is [N, e-1, d_v, d_phi]; the tensor feature-map projection is
 *    [d_k + d_k*d_k, d_phi].
 *  - "io" tensors (k, q, v, gates, y and their gradients) are float32 or
 *    bfloat16 (dtype_io); states, buffers and their gradients are float32.
 *  - The library never allocates: the caller passes workspaces sized by
 *    atlas_mem_workspace_size(). The "saved" workspace is written by the
 *    forward and read by the backward; it must stay untouched in between.
 *  - All work is enqueued on `stream` (a cudaStream_t; NULL = legacy default).
 *  - Return value 0 = success, otherwise an ATLAS_ERR_* code (see
 *    atlas_mem_error_string). Invalid arguments are rejected before any launch.
 */
#ifndef ATLAS_MEM_H
#define ATLAS_MEM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ATLAS_MEM_ABI_VERSION 2

enum AtlasFmapMode { ATLAS_FMAP_OFF = 0, ATLAS_FMAP_ELEMENTWISE = 1, ATLAS_FMAP_TENSOR = 2 };
enum AtlasGateMode { ATLAS_GATE_NONE = 0, ATLAS_GATE_TOKEN = 1, ATLAS_GATE_WINDOW = 2 };
enum AtlasDtype { ATLAS_F32 = 0, ATLAS_BF16 = 1 };

enum AtlasError {
  ATLAS_OK = 0,
  ATLAS_ERR_INVALID_ARG = 1,   /* null pointer / bad enum / inconsistent sizes   */
  ATLAS_ERR_UNSUPPORTED = 2,   /* shape outside the supported envelope            */
  ATLAS_ERR_WORKSPACE = 3,     /* workspace pointer missing or too small          */
  ATLAS_ERR_LAUNCH = 4,        /* a kernel launch failed (cudaGetLastError)        */
  ATLAS_ERR_DEVICE = 5,        /* device-side status word reported a fault         */
  ATLAS_ERR_NOALLOC_TOO_LARGE = 6, /* shape exceeds the fixed scratch of the no-alloc entry */
  ATLAS_ERR_NOALLOC_CAPTURE = 7    /* no-alloc scratch looked up for the first time inside a stream capture */
};

/* Shapes and modes of one call. Mirrors the constructor arguments of
 * RNNMemoryCell / OmegaRNNMemoryCell (rnn_memory.py:167-179, 426-441). */
typedef struct AtlasMemShape {
  int64_t N;          /* batch * heads                                         */
  int64_t T;          /* tokens in this call                                   */
  int32_t d_k;        /* raw key/query width (dim_head)                        */
  int32_t d_phi;      /* feature width (= d_k unless fmap is 'tensor')         */
  int32_t d_v;        /* value width                                           */
  int32_t window;     /* omega window e >= 1                                   */
  int32_t fmap_mode;  /* AtlasFmapMode                                         */
  int32_t fmap_degree;/* polynomial degree g (elementwise: phi = sum x^i)      */
  int32_t gate_mode;  /* AtlasGateMode                                         */
  int32_t momentum;   /* 1 = use_momentum (beta/Z present), 0 = off            */
  int32_t dtype_io;   /* AtlasDtype of k, q, v, gates, y and their gradients   */
  int32_t chunk;      /* internal token chunk; 0 = library default             */
} AtlasMemShape;

/* Forward operands. Optional pointers may be NULL: beta (momentum off),
 * gate (gate_mode NONE), Z0 (zeros), buf_in (zeros), proj (fmap != TENSOR),
 * Z_end (momentum off), buf_out (window 1). */
typedef struct AtlasMemFwd {
  const void* k;       /* [N,T,d_k]  io                                         */
  const void* q;       /* [N,T,d_k]  io                                         */
  const void* v;       /* [N,T,d_v]  io                                         */
  const void* lr;      /* [N,T]      io  eta   (to_lr, rnn_memory.py:645)       */
  const void* decay;   /* [N,T]      io  alpha (to_decay, :646)                 */
  const void* beta;    /* [N,T]      io  (to_momentum, :649)                    */
  const void* gate;    /* [N,T] (TOKEN) or [N,T,e] (WINDOW), io                 */
  const float* S_ref;  /* [N,d_v,d_phi] state the deltas are taken against      */
  const float* S0;     /* [N,d_v,d_phi] carried S                               */
  const float* Z0;     /* [N,d_v,d_phi] carried Z                               */
  const float* buf_in; /* [N,e-1,d_v,d_phi] carried omega buffer                */
  const float* proj;   /* [d_k+d_k^2, d_phi] tensor feature-map projection      */
  void* y;             /* [N,T,d_v]  io  output                                 */
  float* S_end;        /* [N,d_v,d_phi]                                         */
  float* Z_end;        /* [N,d_v,d_phi]                                         */
  float* buf_out;      /* [N,e-1,d_v,d_phi]                                     */
  int* status;         /* optional device-visible status word, see below        */
} AtlasMemFwd;

/* Backward operands: upstream gradients in, input gradients out. Optional
 * upstream gradients (dS_end, dZ_end, dbuf_out) may be NULL (= zeros); output
 * gradients of absent inputs may be NULL and are then not produced. */
typedef struct AtlasMemBwd {
  const void* dy;        /* [N,T,d_v] io                                        */
  const float* dS_end;   /* [N,d_v,d_phi]                                       */
  const float* dZ_end;   /* [N,d_v,d_phi]                                       */
  const float* dbuf_out; /* [N,e-1,d_v,d_phi]                                   */
  void* dk;              /* [N,T,d_k] io                                        */
  void* dq;              /* [N,T,d_k] io                                        */
  void* dv;              /* [N,T,d_v] io                                        */
  void* dlr;             /* [N,T] io                                            */
  void* ddecay;          /* [N,T] io                                            */
  void* dbeta;           /* [N,T] io                                            */
  void* dgate;           /* [N,T] or [N,T,e] io                                 */
  float* dS_ref;         /* [N,d_v,d_phi]                                       */
  float* dS0;            /* [N,d_v,d_phi]                                       */
  float* dZ0;            /* [N,d_v,d_phi]                                       */
  float* dbuf_in;        /* [N,e-1,d_v,d_phi]                                   */
  int* status;           /* optional device-visible status word, see below      */
} AtlasMemBwd;

/* ---- tensor feature map on its own (the 'tensor' mode of
 * PolynomialFeatureMap, rnn_memory.py:106-111,125-130):
 *   phi = [x ; vec(x x^T)] Proj,  x [rows, d_k] bf16, Proj [d_k + d_k^2, d_phi] fp32,
 *   phi [rows, d_phi] bf16 out,
 * on tensor cores without forming the d_k + d_k^2 wide rows. For bf16 io,
 * d_k in {16, 32, 48, 64} and d_phi a multiple of 16 up to 256; other shapes
 * return ATLAS_ERR_UNSUPPORTED (atlas_mem_forward still handles them in its
 * own tensor-mode path). `proj_tiles` is a caller workspace of
 * atlas_fmap_tensor_workspace(d_k, d_phi) bytes: the forward fills it with
 * Proj in bf16 and the backward reads it, so it must stay untouched in
 * between. The backward writes dx [rows, d_k] (bf16) from d phi [rows, d_phi]
 * (bf16); Proj is a fixed buffer and gets no gradient. `status`: optional
 * device status word, as below. The reference computes the same product with
 * einsum + matmul in PolynomialFeatureMap.forward (rnn_memory.py:125-130). */
size_t atlas_fmap_tensor_workspace(int d_k, int d_phi);
int atlas_fmap_tensor_forward(int64_t rows, int d_k, int d_phi, const void* x, const float* proj,
                              void* proj_tiles, void* phi, int* status, void* stream);
int atlas_fmap_tensor_backward(int64_t rows, int d_k, int d_phi, const void* x, const void* proj_tiles,
                               const void* dphi, void* dx, int* status, void* stream);

/* Device status word (`status` in AtlasMemFwd / AtlasMemBwd; NULL = none).
 * Every wait of a kernel for its tensor-core work is bounded. When one runs
 * out, the kernel writes ATLAS_DEVSTAT_MMA_TIMEOUT to *status, lets its copies
 * and tensor-core work in flight drain (again bounded), releases its tensor
 * memory and returns without writing the rest of its results; the call's
 * outputs are then invalid. The caller zeroes the word (device memory, or
 * pinned host memory the device can reach) and reads it once the work has
 * finished, for example with atlas_mem_read_status. The library never clears
 * it, so one word can collect the status of many calls. */
#define ATLAS_DEVSTAT_MMA_TIMEOUT 1

/* Synchronises `stream`, reads *status (a device or device-visible pointer)
 * and returns ATLAS_ERR_DEVICE if it is nonzero, ATLAS_OK otherwise
 * (ATLAS_ERR_LAUNCH if the synchronisation or the read failed). The word is
 * left as it is. No reference counterpart (the reference has no device-side
 * error reporting). */
int atlas_mem_read_status(const int* status, void* stream);

/* Self test of the bounded-wait path: one CTA initialises a barrier that
 * nothing ever arrives on and waits on it for `polls` polls through the same
 * wait-and-report code the tensor-core kernels use, so *status receives
 * ATLAS_DEVSTAT_MMA_TIMEOUT. No tensor-core work is issued and no tensor
 * memory is held, so the timeout is harmless and the context stays usable.
 * polls must be in [1, 1<<20]. No reference counterpart. */
int atlas_mem_selftest_wait_timeout(int* status, int polls, void* stream);

/* Library version / ABI check. */
int atlas_mem_abi_version(void);

/* Human-readable text for an AtlasError code (static storage). */
const char* atlas_mem_error_string(int code);

/* Workspace sizes in bytes for a shape: `saved` lives from forward to
 * backward, `fwd_scratch` / `bwd_scratch` only during one call. Any output
 * pointer may be NULL. Replaces the per-call torch.empty allocations of
 * atlas_omega_autograd.py:125-134,175-184. */
int atlas_mem_workspace_size(const AtlasMemShape* shape, size_t* saved,
                             size_t* fwd_scratch, size_t* bwd_scratch);

/* Forward pass (AtlasOmegaFunction.forward, atlas_omega_autograd.py:98-153;
 * semantics of OmegaRNNMemoryCell._forward_impl, rnn_memory.py:655-730). */
int atlas_mem_forward(const AtlasMemShape* shape, const AtlasMemFwd* fwd,
                      void* saved, size_t saved_bytes,
                      void* scratch, size_t scratch_bytes, void* stream);

/* Forward pass that allocates nothing and takes no workspace. No counterpart
 * in the reference: it is for callers that own only their input and output
 * buffers and cannot call cudaMalloc -- for example a plugin slot in a host
 * framework that hands over tensors but no workspace, or a serving loop whose
 * device memory is fully reserved by its own pool.
 *  - Scratch lives in one fixed device array of atlas_mem_noalloc_scratch_bytes()
 *    (32 MiB) inside the library; every GPU that loads the library holds it
 *    until the process exits. Shapes whose forward workspace
 *    (atlas_mem_workspace_size's `saved`) exceeds it are rejected with
 *    ATLAS_ERR_NOALLOC_TOO_LARGE before anything is launched.
 *  - Every call looks up the array's device address with the current device
 *    (nothing is cached, so a context reset is harmless). The first lookup on
 *    a device loads the library's kernels there, which CUDA refuses inside a
 *    stream capture: make the first call on each device before any capture
 *    (a first call made during capture returns ATLAS_ERR_NOALLOC_CAPTURE).
 *  - All calls share the one array and it keeps the last call's contents:
 *    calls whose work overlaps on the GPU (other streams, other host threads)
 *    race with each other. Nothing in it needs to start at zero.
 *  - Same operands and results as atlas_mem_forward; no backward can follow
 *    (nothing is kept for it). Calls no cudaMalloc, cudaFree or allocating
 *    library routine. */
int atlas_mem_forward_noalloc(const AtlasMemShape* shape, const AtlasMemFwd* fwd, void* stream);
/* Size in bytes of the fixed scratch array used by atlas_mem_forward_noalloc. */
size_t atlas_mem_noalloc_scratch_bytes(void);

/* One decoding step (shape->T == 1) without workspaces: the token's memory
 * update and read-out in a single streaming kernel, for inference loops that
 * call the cell one token at a time with the state carried (the reference's
 * generate, rnn_transformer.py:864-904, through OmegaRNNMemoryCell.forward with
 * seq_len 1; semantics rnn_memory.py:655-730 at T = 1):
 *   delta = S_ref phi(k) - v,  g = window sum over [buf_in, delta phi(k)^T],
 *   Z_end = beta Z0 + g,  S_end = clamp(alpha S0 - eta Z_end, -100, 100)
 *   (without momentum S_end = clamp(alpha S0 - eta g)),  y = S0 phi(q),
 *   buf_out = buf_in shifted by one entry with delta phi(k)^T appended.
 * Same operands and results as atlas_mem_forward with T = 1; no backward can
 * follow. d_phi, d_v <= 256; the tensor feature map is not handled
 * (ATLAS_ERR_UNSUPPORTED: use atlas_mem_forward). buf_out must not alias
 * buf_in. Allocates nothing. */
int atlas_mem_decode_step(const AtlasMemShape* shape, const AtlasMemFwd* fwd, void* stream);

/* Backward pass (AtlasOmegaFunction.backward, atlas_omega_autograd.py:155-204;
 * gradients of the PyTorch path's autograd). `fwd` must hold the same
 * forward operands (outputs may be NULL) and `saved` the forward's workspace. */
int atlas_mem_backward(const AtlasMemShape* shape, const AtlasMemFwd* fwd,
                       const AtlasMemBwd* bwd, const void* saved, size_t saved_bytes,
                       void* scratch, size_t scratch_bytes, void* stream);

/* ---- sequence-parallel pieces (no reference counterpart: the reference has
 * no distributed code). A rank holding tokens [t_lo, t_hi) of a longer
 * sequence runs *_local, exchanges the per-unit segment transforms with the
 * other ranks (the host does this over NCCL), then runs *_finish with the
 * incoming carry. The segment transform of a rank is
 *   (S, Z) -> (a*S + b*Z + dS, c*Z + dZ)
 * with per-unit scalars coef[N,3] = (a, b, c) and matrices dS, dZ [N,d_v,d_phi].
 * Requires window == 1 (no cross-rank halo). */
int atlas_mem_forward_local(const AtlasMemShape* shape, const AtlasMemFwd* fwd,
                            void* saved, size_t saved_bytes, void* scratch,
                            size_t scratch_bytes, float* seg_coef, float* seg_dS,
                            float* seg_dZ, void* stream);
/* Completes the forward given the incoming carry in fwd->S0 / fwd->Z0 (S_ref
 * stays the call-start state of the whole sequence). */
int atlas_mem_forward_finish(const AtlasMemShape* shape, const AtlasMemFwd* fwd,
                             void* saved, size_t saved_bytes, void* scratch,
                             size_t scratch_bytes, void* stream);
/* Copies the unclamped final state S_T of the last forward (held in `saved`)
 * to out[N,d_v,d_phi]; the rank holding the end of the sequence uses it for
 * the clamp mask of dS_end (rnn_memory.py:701). */
int atlas_mem_final_state_raw(const AtlasMemShape* shape, const void* saved, size_t saved_bytes, float* out,
                              void* stream);
/* Backward segment transform of this rank, computed from zero adjoint:
 *   (FS, FZ) -> (a*FS + dFS, b*FS + c*FZ + dFZ)   coef[N,3] = (a, b, c). */
int atlas_mem_backward_local(const AtlasMemShape* shape, const AtlasMemFwd* fwd,
                             const AtlasMemBwd* bwd, const void* saved, size_t saved_bytes,
                             void* scratch, size_t scratch_bytes, float* seg_coef,
                             float* seg_dS, float* seg_dZ, void* stream);
/* Completes the backward given the adjoint arriving from later ranks in
 * bwd->dS_end / bwd->dZ_end (the last rank passes the true upstream gradients,
 * apply_clamp_mask = 1 there only). dS_ref receives this rank's partial sum. */
int atlas_mem_backward_finish(const AtlasMemShape* shape, const AtlasMemFwd* fwd,
                              const AtlasMemBwd* bwd, const void* saved, size_t saved_bytes,
                              void* scratch, size_t scratch_bytes, int apply_clamp_mask,
                              void* stream);

/* Composes the gathered segment transforms of all `world` ranks (the host-side
 * step of the carry exchange, done on the device in one pass). seg is
 * [world][record_len] floats; a rank's record is coef [N,3] padded to a
 * multiple of 4 floats, then dS [N,d2], then dZ [N,d2] (the buffers
 * *_local fill). Forward (backward = 0): S0 / Z0 (Z0 may be NULL = 0) through
 * ranks 0..world-1; in_S / in_Z receive the carry entering `rank`, out_S the
 * unclamped S_T, out_S_clamped clamp(S_T, -100, 100), out_Z Z_T. Backward:
 * S0 / Z0 are the summed dS_end / dZ_end (NULL = 0), dS_end masked where S_T
 * (NULL = no mask) lies outside [-100, 100], composed through ranks
 * world-1..0; in_* receive the adjoint arriving at the end of `rank`'s
 * segment, out_S / out_Z the adjoint at the sequence start (dS0 / dZ0).
 * Any output may be NULL. */
int atlas_mem_compose_carries(const float* seg, int64_t record_len, int world, int rank, int64_t N, int64_t d2,
                              int backward, const float* S0, const float* Z0, const float* S_T, float* in_S,
                              float* in_Z, float* out_S, float* out_S_clamped, float* out_Z, void* stream);

/* The three depthwise convolutions in front of q, k and v in the memory cells
 * (rnn_memory.py:196-202,334-340: Conv1d(C, C, K, padding=K/2, groups=C,
 * bias=False) over the sequence, first T outputs kept), in one pass over x in
 * its [B, T, C] layout: y_m[b,t,c] = sum_j w_m[c,j] x[b, t+j-K/2, c] (zero
 * outside the sequence) for m = q, k, v. w_* are fp32 [C, K] (the Conv1d weight
 * [C, 1, K]); x in dtype_x, outputs in dtype_y (ATLAS_F32 / ATLAS_BF16);
 * fp32 accumulation. 2 <= K <= 8, B <= 65535. */
int atlas_dwconv3_forward(const void* x, int dtype_x, const float* w_q, const float* w_k, const float* w_v, int K,
                          void* y_q, void* y_k, void* y_v, int dtype_y, int64_t B, int64_t T, int64_t C,
                          void* stream);
/* Its backward: dx (dtype_x, [B, T, C]; the sum over the three convolutions)
 * and dw fp32 [3, C, K] (q, k, v weight gradients; zeroed here, then summed). */
int atlas_dwconv3_backward(const void* x, int dtype_x, const float* w_q, const float* w_k, const float* w_v, int K,
                           const void* dy_q, const void* dy_k, const void* dy_v, int dtype_y, void* dx,
                           float* dw, int64_t B, int64_t T, int64_t C, void* stream);

/* Head preparation of the memory cells: the projection output t [B, T, H*d]
 * is split into heads, RMS-normalised per head with gain gamma [H, d] when
 * gamma is given (MultiheadRMSNorm, rnn_memory.py:139-147: x / max(||x|| d^-1/2,
 * 1e-8) * gamma[h]) and written as out [B*H, T, d_out] with zero columns
 * d..d_out-1. d in {32, 64, 96, 128}; dtypes ATLAS_F32 / ATLAS_BF16. */
int atlas_head_prep_forward(const void* t, int dtype_in, const float* gamma, void* out, int dtype_out, int64_t B,
                            int64_t T, int H, int d, int d_out, void* stream);
/* Its backward: grad_t [B, T, H*d] (dtype_in) from grad_out [B*H, T, d_out]
 * (its first d columns), and grad_gamma [H, d] fp32 (zeroed here; may be NULL;
 * needs gamma). */
int atlas_head_prep_backward(const void* t, int dtype_in, const float* gamma, const void* grad_out, int dtype_out,
                             void* grad_t, float* grad_gamma, int64_t B, int64_t T, int H, int d, int d_out,
                             void* stream);

/* Device self-check of the tensor-core (tcgen05) GEMM building block used by
 * the fused kernels: D[128,N] = A[128,K] * B^T with A given as [128][K]
 * (a_mn_major = 0) or [K][128] (1), B as [N][K] (b_mn_major = 0) or [K][N] (1);
 * bf16 operands, fp32 D. *status (device int, zeroed by the caller) becomes
 * nonzero if the bounded completion wait timed out. No reference counterpart. */
int atlas_mem_selftest_umma(const void* A, const void* B, float* D, int N, int K, int a_mn_major,
                            int b_mn_major, int* status, void* stream);

/* ---- measurement hooks (no reference counterpart: the reference only prints
 * wall-clock times, tests/test_atlas_cuda.py:270-284). Every kernel launch is
 * counted; with timing enabled each launch is bracketed by CUDA events recorded
 * on its own stream, summed per kernel when read. */
/* Reset counters and turn per-launch event timing on (1) or off (0). */
int atlas_mem_profile_enable(int on);
/* Total event-timed milliseconds and timed launches of one kernel since the
 * last reset (waits for the pending events). */
int atlas_mem_profile_read(int kernel_id, double* total_ms, long long* launches);
/* Kernel launches issued since the last reset (timed or not). */
long long atlas_mem_launch_count(void);
/* Number of kernel ids and the name of one. */
int atlas_mem_kernel_count(void);
const char* atlas_mem_kernel_name(int kernel_id);

/* ---- scalar-gated scan (drop-in for assoc_scan.AssocScan) -----------------
 * The reference's legacy OmegaNeuralMemory (omega.py:262-315) and the Titans
 * paths call the third-party AssocScan as AssocScan()(gates, inputs, prev=...,
 * remove_prev=...) (rnn_memory.py:34,189,363-379; omega.py:315): over dim 1,
 *   h_t = gates[b,t] * h_{t-1} + inputs[b,t,...],  h_0 = prev[b,...] (or 0),
 * outputs h_1..h_T, with prev prepended (T + 1 outputs) when remove_prev is
 * false. gates [B,T] fp32; inputs / outputs [B,T,D] (trailing dims flattened)
 * in fp32 or bf16 (dtype_io), fp32 accumulation; prev [B,D] fp32 or NULL. */
int atlas_scan_forward(const float* gates, const void* inputs, const float* prev, void* out, int64_t B,
                       int64_t T, int64_t D, int dtype_io, int remove_prev, void* stream);
/* Backward of atlas_scan_forward. out is the forward output (with prev
 * prepended when remove_prev was false), dout its gradient (same layout and
 * dtype). d_gates [B,T] fp32 (required; it is accumulated over D, zeroed
 * here), d_inputs [B,T,D] in dtype_io, d_prev [B,D] fp32 or NULL. */
int atlas_scan_backward(const float* gates, const void* out, const float* prev, const void* dout,
                        float* d_gates, void* d_inputs, float* d_prev, int64_t B, int64_t T, int64_t D,
                        int dtype_io, int remove_prev, void* stream);

/* ---- right-affine matrix scan: the GPU counterpart of the reference's
 * affine_associative_scan (atlas_pytorch/affine_scan.py:36-160; composition
 * rule _assoc_compose_affine :7-33):
 *   H_t = H_{t-1} A_t + B_t,  H_{-1} = prev (NULL = zeros),
 * A [N,T,D,D], B [N,T,R,D], prev [N,R,D], all fp32. out [N,T+1,R,D] with
 * prev first when prev is given and remove_prev is 0, else [N,T,R,D]
 * (the reference's remove_prev=True keeps the T states). R and D multiples of
 * 8 up to 128. The backward takes the forward's out and its gradient d_out
 * (same layout) and writes d_A, d_B (required) and d_prev (when prev is
 * given). */
int atlas_affine_scan_forward(const float* A, const float* B, const float* prev, float* out, int64_t N,
                              int64_t T, int R, int D, int remove_prev, void* stream);
int atlas_affine_scan_backward(const float* A, const float* prev, const float* out, const float* d_out,
                               float* d_A, float* d_B, float* d_prev, int64_t N, int64_t T, int R, int D,
                               int remove_prev, void* stream);

/* ---- legacy OmegaNeuralMemory per-parameter update (omega.py:262-315) ----
 * One fused pass over surprises s [B,T,D] (B = batch*heads, T = chunks, D =
 * the parameter's elements flattened), replacing the momentum assoc_scan
 * (omega.py:262-268), the omega gate (:276-283), the window sum with the
 * carried __omega_buf (:285-298, _sliding_sum_along_n :24-33) and the decay
 * assoc_scan with remove_prev=False (:315):
 *   m_t = beta_t m_{t-1} + s_t  (m_0 = last_momentum; beta NULL: m_t = s_t)
 *   g_t = gate_t m_t            (gate NULL: g_t = m_t)
 *   w_t = sum_{j<window} g_{t-j}, g_{-1}.. from buf_in [B,window-1,D] (NULL = zeros)
 *   h_t = keep_t h_{t-1} + w_t  (keep = 1 - decay_factor; h_0 = last_update)
 * out [B,T+1,D] = h_0..h_T when last_update is given, else [B,T,D] = h_1..h_T;
 * momentum_last [B,D] = m_T (may be NULL); buf_out [B,window-1,D] = the last
 * window-1 entries of [buf_in; g]; momentum_all [B,T,D] fp32 keeps m for the
 * backward (needed there when beta is given). Scalars [B,T] fp32, states fp32,
 * s / out / d_out / d_surprise in dtype_io. window <= 16, B <= 65535. */
int atlas_omega_store_forward(const float* beta, const void* surprise, const float* last_momentum,
                              const float* gate, const float* buf_in, const float* keep,
                              const float* last_update, void* out, float* momentum_all,
                              float* momentum_last, float* buf_out, int64_t B, int64_t T, int64_t D,
                              int window, int dtype_io, void* stream);
/* Backward of atlas_omega_store_forward: d_out like out; d_momentum_last,
 * d_buf_out optional upstream gradients. d_beta, d_gate, d_keep [B,T] are
 * zeroed here and accumulated over D; d_last_momentum, d_last_update [B,D] and
 * d_buf_in [B,window-1,D] may be NULL. */
int atlas_omega_store_backward(const float* beta, const void* surprise, const float* last_momentum,
                               const float* gate, const float* keep, const float* last_update, const void* out,
                               const float* momentum_all, const void* d_out, const float* d_momentum_last,
                               const float* d_buf_out, void* d_surprise, float* d_beta, float* d_gate,
                               float* d_keep, float* d_last_momentum, float* d_last_update, float* d_buf_in,
                               int64_t B, int64_t T, int64_t D, int window, int dtype_io, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ATLAS_MEM_H */

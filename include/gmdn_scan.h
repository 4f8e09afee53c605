/*
 * gmdn_scan.h -- C ABI of the B200 (sm_100a) chunkwise gated fast-weight
 * state scan: delta, muon and adam inner rules, forward and backward.
 *
 * Two layers of the reference are replaced:
 *
 *   1. the phase-2 state scan, fast_scan.py:403 `fast_state_scan(U, K, a, b,
 *      m, n, rule, ns)` and its autograd Function `_TritonScan`
 *      (fast_scan.py:334-396) -> gmdn_scan_fwd / gmdn_scan_bwd;
 *   2. the mixer core around it, train_ablation.py:142-187 (phase 1
 *      intra-chunk products, the scan, phase 3 output) -> gmdn_chunk_fwd /
 *      gmdn_chunk_bwd.
 *
 * Conventions
 *   - All tensors are dense, row-major, contiguous, on the current CUDA device.
 *   - Scan tensors: U, K, S (B, H, N, dh, dh) fp32; gates a, b, m, n (B, H, N)
 *     fp32.  Each state is stored [dv, dk] (rows are the value dimension), as
 *     in the reference.  The forward writes the PRE-update states S_0..S_{N-1}.
 *   - Mixer tensors: q, k, v, o and their gradients (B, H, T, dh) bf16 (raw
 *     bits as uint16_t); gates alpha, beta, mu, nu (B, H, T) fp32.
 *   - rule: 0 = delta, 1 = muon, 2 = adam.  ns: Newton-Schulz steps (muon).
 *   - precision: GMDN_PREC_IEEE = exact fp32 products (the reference's
 *     set_precision('ieee')); GMDN_PREC_FAST = tensor-core products (the
 *     reference's default 'tf32' mode).
 *   - Nothing is allocated inside: the caller passes device buffers of the
 *     sizes the *_bytes() queries return.  No host synchronisation; all work is
 *     enqueued on `stream` (a cudaStream_t, 0 = legacy default stream).
 *   - Every entry point returns 0 on success or a GMDN_ERR_* code; the message
 *     of the calling thread's last failure is gmdn_last_error_string().
 *   - The functions keep no state between calls and may be called from any
 *     host thread.
 */
#ifndef GMDN_SCAN_H_
#define GMDN_SCAN_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  GMDN_OK = 0,
  GMDN_ERR_INVALID = 1,     /* bad shape, rule, ns or null pointer */
  GMDN_ERR_UNSUPPORTED = 2, /* valid but not built (dh, chunk, precision) */
  GMDN_ERR_WORKSPACE = 3,   /* workspace smaller than required */
  GMDN_ERR_CUDA = 4,        /* a CUDA launch or device query failed */
  GMDN_ERR_DEVICE = 5       /* a kernel reported a failure through its status word */
};

enum { GMDN_PREC_IEEE = 0, GMDN_PREC_FAST = 1 };

/* Version of this ABI; bumped on any signature change. */
int gmdn_abi_version(void);

/* Message for the calling thread's most recent failed call ("" if none). */
const char* gmdn_last_error_string(void);

/* ---- phase-2 state scan: fast_scan.py:403 fast_state_scan ---------------- */

/* Bytes of `saved` the forward fills for the backward (the pre-update M and V
 * histories for muon / adam; replaces the M_all / V_all tensors that
 * fast_scan.py:367-368 allocates). */
size_t gmdn_scan_saved_bytes(int B, int H, int N, int dh, int rule);

/* Scratch bytes for gmdn_scan_fwd / gmdn_scan_bwd.  The first 256 bytes hold
 * the device status word that gmdn_chunk_status reads after a call. */
size_t gmdn_scan_workspace_bytes(int B, int H, int N, int dh, int rule, int ns,
                                 int precision);

/* Forward: S_out <- pre-update states.  Replaces _TritonScan.forward
 * (fast_scan.py:360-377) and _scan_fwd_kernel (fast_scan.py:206-248).
 * precision GMDN_PREC_FAST (the reference's tf32 default) with rule 0 (delta)
 * at dh 128 runs the tensor-core scan (split-bf16 products, ~16 significant
 * bits per operand, within 1e-4 of the fp32 recurrence); every other case, and
 * GMDN_PREC_IEEE, runs exact fp32 FMAs.  gmdn_scan_bwd follows the same rule. */
int gmdn_scan_fwd(const float* U, const float* K, const float* a, const float* b,
                  const float* m, const float* n, float* S_out, void* saved,
                  void* workspace, size_t workspace_bytes, int B, int H, int N,
                  int dh, int rule, int ns, int precision, void* stream);

/* Backward: cotangents of U, K, a, b, m, n for the cotangent gS of the state
 * stack.  Gates the rule does not read get zeros (the reference's Triton
 * backward leaves them uninitialised, fast_scan.py:386-389).  Replaces
 * _TritonScan.backward (fast_scan.py:380-396) and _scan_bwd_kernel
 * (fast_scan.py:269-331). */
int gmdn_scan_bwd(const float* U, const float* K, const float* a, const float* b,
                  const float* m, const float* n, const float* S_all,
                  const void* saved, const float* gS, float* dU, float* dK,
                  float* da, float* db, float* dm, float* dn, void* workspace,
                  size_t workspace_bytes, int B, int H, int N, int dh, int rule,
                  int ns, int precision, void* stream);

/* Size of the device scratch array gmdn_scan_fwd_noalloc uses: 16 MiB, held
 * by every GPU that loads this library until the process exits. */
#define GMDN_NOALLOC_SCRATCH_BYTES (16u * 1024u * 1024u)

/* gmdn_scan_fwd without a workspace: same arguments and results, but its
 * scratch is a fixed device array inside this library, so the call allocates
 * nothing.  It always runs the exact-fp32 scan (the kernel that needs the
 * scratch), for either `precision`.  No counterpart in the reference (its
 * Triton wrapper allocates with torch, fast_scan.py:366-368).
 *
 * For callers that cannot allocate device memory: a runtime that owns every
 * device buffer and hands a foreign call only its operands and results (a
 * framework's custom-call hook, a fixed-pool embedded runtime).  A cudaMalloc
 * from inside such a call goes around that runtime's memory pool: it can fail
 * once the pool has reserved the GPU, and cudaMalloc / cudaFree may
 * synchronise the device and stall the caller's other streams.
 *
 * Limit: B*H*6*dh*dh*4 bytes <= GMDN_NOALLOC_SCRATCH_BYTES, i.e. at most 42
 * (b,h) pairs at dh 128, 170 at dh 64, 682 at dh 32, 2730 at dh 16; larger
 * calls return GMDN_ERR_WORKSPACE with the limit in the message.  The caller
 * still passes inputs, S_out and (muon / adam) `saved`.
 *
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture.  Every call on a device shares the one array,
 * which keeps the last call's contents (the kernel clears what must start at
 * zero): calls that overlap on the GPU, from two streams or two host threads,
 * race on it and give wrong results, so keep them in order on one stream.
 * The looked-up address lives as long as the device's context: a reset of the
 * device (cudaDeviceReset, or a primary-context reset) unloads this library's
 * device code and leaves the address stale, so do not call this entry point
 * on a device after resetting it in the same process. */
int gmdn_scan_fwd_noalloc(const float* U, const float* K, const float* a,
                          const float* b, const float* m, const float* n,
                          float* S_out, void* saved, int B, int H, int N, int dh,
                          int rule, int ns, int precision, void* stream);

/* ---- mixer core: train_ablation.py:142-187 ------------------------------- */

/* Bytes of `saved` the chunk forward fills for the chunk backward. */
size_t gmdn_chunk_saved_bytes(int B, int H, int T, int dh, int chunk, int rule,
                              int ns, int precision);

/* Scratch bytes for gmdn_chunk_fwd / gmdn_chunk_bwd. */
size_t gmdn_chunk_workspace_bytes(int B, int H, int T, int dh, int chunk, int rule,
                                  int ns, int precision);

/* Forward of phases 1-3: o = (q - A k) S^T + A v per chunk with
 * A = tril(q k^T) * beta (train_ablation.py:160-167, 184-187), the states S
 * from the scan over Kw = k^T diag(w) k, Uv = v^T diag(w) k and the chunk
 * gate products (train_ablation.py:150-182).  `nu` is read only by rule 2 and
 * may be NULL otherwise. */
int gmdn_chunk_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                   const float* alpha, const float* beta, const float* mu,
                   const float* nu, uint16_t* o, void* saved, void* workspace,
                   size_t workspace_bytes, int B, int H, int T, int dh, int chunk,
                   int rule, int ns, int precision, void* stream);

/* Backward of gmdn_chunk_fwd for the output cotangent dO.  Writes the
 * cotangents of q, k, v (bf16) and of each gate (fp32); dnu may be NULL
 * unless rule == 2.  Gates a rule does not read get zeros. */
int gmdn_chunk_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                   const float* alpha, const float* beta, const float* mu,
                   const float* nu, const uint16_t* dO, const void* saved,
                   uint16_t* dq, uint16_t* dk, uint16_t* dv, float* dalpha,
                   float* dbeta, float* dmu, float* dnu, void* workspace,
                   size_t workspace_bytes, int B, int H, int T, int dh, int chunk,
                   int rule, int ns, int precision, void* stream);

/* Same as gmdn_chunk_fwd / gmdn_chunk_bwd with the activation dtype chosen at
 * run time: io_f32 = 0 for bf16 q/k/v/o/dO/dq/dk/dv (the autocast-bf16 trainer,
 * train_ablation.py:465-467), 1 for fp32 (the fp32 runs the 1e-4 parity bar
 * is stated on).  Pointers are untyped for that reason. */
int gmdn_chunk_fwd_ex(const void* q, const void* k, const void* v, const float* alpha,
                      const float* beta, const float* mu, const float* nu, void* o,
                      void* saved, void* workspace, size_t workspace_bytes, int B, int H,
                      int T, int dh, int chunk, int rule, int ns, int precision, int io_f32,
                      void* stream);

int gmdn_chunk_bwd_ex(const void* q, const void* k, const void* v, const float* alpha,
                      const float* beta, const float* mu, const float* nu, const void* dO,
                      const void* saved, void* dq, void* dk, void* dv, float* dalpha,
                      float* dbeta, float* dmu, float* dnu, void* workspace,
                      size_t workspace_bytes, int B, int H, int T, int dh, int chunk,
                      int rule, int ns, int precision, int io_f32, void* stream);

/* Buffer sizes for gmdn_chunk_fwd_ex / gmdn_chunk_bwd_ex with the given
 * activation dtype (the layout of `saved` depends on it: the tensor-core path
 * keeps the states in bf16). */
size_t gmdn_chunk_saved_bytes_ex(int B, int H, int T, int dh, int chunk, int rule,
                                 int ns, int precision, int io_f32);
size_t gmdn_chunk_workspace_bytes_ex(int B, int H, int T, int dh, int chunk, int rule,
                                     int ns, int precision, int io_f32);

/* Reads the device status word the last chunk or scan call on this workspace
 * left (synchronises `stream`): GMDN_OK, or GMDN_ERR_DEVICE when a kernel gave
 * up a bounded wait.  No reference counterpart (the reference has no device-side
 * failure reporting). */
int gmdn_chunk_status(const void* workspace, void* stream);

/* Mixer prologue, replaces train_ablation.py:124-140 after the two
 * projections: qkv = silu(conv(u)) with u = self.qkv(x) (B, T, 3D) and conv
 * the depthwise causal Conv1d (kernel 4, padding 3, first T outputs; weight
 * (3D, 1, 4) and bias (3D) fp32); q and k L2-normalised per head over dh
 * (F.normalize, eps 1e-12), v as is, all (B, H, T, dh); g = sigmoid(gl) with
 * gl = self.gates(x) (B, T, nG*H) into (nG, B, H, T).  fp32 arithmetic, I/O in
 * bf16 (io_f32 0) or fp32 (1); dh 32, 64 or 128; n_gates 3 or 4; B*T*3D
 * below 2^31; tensor pointers 16-byte aligned.  The backward takes dq, dk, dv
 * (B, H, T, dh) and dg (nG, B, H, T) and writes du (B, T, 3D), dgl
 * (B, T, nG*H) and the fp32 conv gradients dconv_w (3D*4), dconv_b (3D)
 * (overwritten, not accumulated). */
int gmdn_mixer_prologue_fwd(const void* u, const float* conv_w, const float* conv_b,
                            const void* gl, void* q, void* k, void* v, void* g, int B, int T,
                            int H, int dh, int n_gates, int io_f32, void* stream);
int gmdn_mixer_prologue_bwd(const void* u, const float* conv_w, const float* conv_b,
                            const void* gl, const void* dq, const void* dk, const void* dv,
                            const void* dg, void* du, float* dconv_w, float* dconv_b, void* dgl,
                            int B, int T, int H, int dh, int n_gates, int io_f32, void* stream);

/* Mixer epilogue, replaces train_ablation.py:188-189 up to the output
 * projection: `o = self.norm(o).to(x.dtype)` with norm = nn.RMSNorm(dh), then
 * `o.transpose(1, 2).reshape(B, T, D)`.  o (B, H, T, dh), weight (dh) fp32,
 * y (B, T, H * dh).  Per row: upcast to fp32, x * rsqrt(mean(x^2) + eps) *
 * weight, rounded to the input dtype, stored in the output dtype (torch's
 * rms_norm for bf16 / fp32 input; eps < 0 selects its default FLT_EPSILON).
 * in_f32 / out_f32: 1 = fp32, 0 = bf16.  dh must be 32, 64 or 128; pointers
 * 16-byte aligned.  The backward takes dy in the output dtype and writes
 * d_o (input dtype) and dweight (fp32; overwritten, not accumulated). */
int gmdn_head_rmsnorm_fwd(const void* o, const float* weight, void* y, int B, int H, int T,
                          int dh, float eps, int in_f32, int out_f32, void* stream);
int gmdn_head_rmsnorm_bwd(const void* o, const float* weight, const void* dy, void* d_o,
                          float* dweight, int B, int H, int T, int dh, float eps, int in_f32,
                          int out_f32, void* stream);

/* Failure-detection self-test (diagnostic; no reference counterpart): launches
 * one CTA whose bounded mbarrier wait -- the same wait the kernels use -- can
 * never complete, with a limit of limit_ns (clamped to [1 ms, 2 s]).  The wait
 * gives up, ORs 1 into the device word *status and the kernel returns; the
 * context stays usable.  GMDN_OK when the launch succeeded (read *status after
 * synchronising `stream`). */
int gmdn_selftest_wait_timeout(uint32_t* status, uint64_t limit_ns, void* stream);

/* Number of kernels this library has enqueued in this process (diagnostic;
 * no reference counterpart). */
uint64_t gmdn_kernel_launches(void);

/* How gmdn_chunk_bwd(_ex) splits the delta backward on the tensor-core path
 * (diagnostic for benchmarks; no reference counterpart): with fewer
 * (b, h) sequences than SMs, one cooperative launch runs the reverse chains
 * and, on the SMs they leave, the token gradients of the first n tiles
 * (chunk-heads) in the order the chains finish them; a second launch does
 * the other B*H*(T/chunk) - n.  Returns n, or 0 where the backward is the
 * two plain launches. */
int gmdn_chunk_bwd_fused_tiles(int B, int H, int T, int dh, int chunk, int rule, int precision,
                               int io_f32);

/* Per-launch timing for benchmarks (diagnostic; no reference counterpart).
 * gmdn_prof_enable(1) brackets every subsequent kernel launch with two CUDA
 * events on its stream; gmdn_prof_report() waits for the recorded events and
 * returns a JSON object {"kernel": [total_ms, launches], ...} of everything
 * recorded since the previous report (the string stays valid until the next
 * call). */
void gmdn_prof_enable(int on);
const char* gmdn_prof_report(void);

#ifdef __cplusplus
}
#endif

#endif /* GMDN_SCAN_H_ */

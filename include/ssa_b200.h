/*
 * ssa_b200.h — C ABI of the B200 (sm_100a) SSA attention library (libssa_b200.so).
 *
 * SSA ("Softmax-Substituted Attention") replaces the softmax logit s = scale * q.k with
 *     t(s) = n * sign(s) * log1p(b * |s|),   P = softmax_j(t),   O = P V
 * (reference: training/train/train_ssa_triton/SSA/ssa_triton_kernel.py:96-113).
 *
 * Conventions shared by every entry point
 *   - Tensors are addressed as [B, H, N, D] with element strides {sB, sH, sN} and a
 *     unit stride on D (the reference kernels take 4 strides, ssa_triton_kernel.py:160-164;
 *     a D stride other than 1 is rejected with SSA_ERR_BAD_STRIDE).
 *   - Packed documents ("varlen"): pass cu_seqlens (int32, device, ndoc+1 entries) and
 *     B = ndoc; every tensor is then [T, H, D] given as {sB = 0, sH, sN} with N = T (total
 *     tokens) and max_seqlen = the longest document. lse / delta are [H, T] in that mode.
 *     Padded packing (documents separated by padding rows) adds cu_seqlens_padded.
 *   - ssa_n is a device pointer to 1 float (reference: 0-d tensor, ssa_triton_attention.py:101)
 *     or to Hq floats (per-head n) when n_per_head != 0; ssa_b is a device pointer to 1 float.
 *     Both are read on the device, so no host synchronisation happens.
 *   - lse is the base-2 normaliser M = log2(sum_j exp2(t_j * log2 e)), fp32, [B, Hq, N]
 *     contiguous (ssa_triton_kernel.py:248-255).
 *   - Entry points that launch work first make the device owning the tensors current on the
 *     calling thread (cudaSetDevice), so a thread that has not used CUDA yet works too.
 *   - All launches are asynchronous on `stream` (a cudaStream_t). Nothing here allocates
 *     device memory: scratch space is the caller's `workspace` (size from the *_workspace_size
 *     query). Entry points return an ssa_status_t; on error ssa_last_error() describes it.
 */
#ifndef SSA_B200_H
#define SSA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  SSA_OK = 0,
  SSA_ERR_BAD_SHAPE = 1,      /* B/H/N/D or GQA ratio invalid (reference asserts, ssa_triton_kernel.py:753,764) */
  SSA_ERR_BAD_STRIDE = 2,     /* D stride != 1, or a stride/base not 16-byte aligned where TMA needs it */
  SSA_ERR_UNSUPPORTED = 3,    /* dtype / head dim not supported */
  SSA_ERR_WORKSPACE = 4,      /* workspace missing or too small */
  SSA_ERR_LAUNCH = 5,         /* CUDA launch error (cudaGetLastError) */
  SSA_ERR_DEVICE_TIMEOUT = 6, /* a bounded device-side wait expired (see ssa_device_status) */
  SSA_ERR_NULL = 7,           /* a required pointer is NULL */
  SSA_ERR_CUDA = 8            /* other CUDA runtime error */
} ssa_status_t;

typedef enum { SSA_DTYPE_F32 = 0, SSA_DTYPE_F16 = 1, SSA_DTYPE_BF16 = 2 } ssa_dtype_t;

/* Strided [B, H, N, D] view: element strides for B, H, N (D stride is 1). */
typedef struct {
  void* ptr;
  int64_t sB, sH, sN;
} ssa_tensor_t;

/* Problem description shared by forward and backward. */
typedef struct {
  int32_t dtype;        /* ssa_dtype_t of q/k/v/o/do/dq/dk/dv */
  int32_t B, Hq, Hkv, N, D;
  int32_t causal;       /* reference: causal flag, ssa_triton_kernel.py:732 */
  float softmax_scale;  /* reference: softmax_scale (1/sqrt(D), optionally / layer_number) */
  const float* ssa_n;   /* device, 1 or Hq floats */
  int32_t n_per_head;
  const float* ssa_b;   /* device, 1 float */
  const int32_t* cu_seqlens; /* device, B+1 entries, or NULL for dense [B,H,N,D] */
  int32_t max_seqlen;        /* longest document when cu_seqlens != NULL */
  /* Optional (packed mode only): device, B+1 entries, the row where each document starts when
   * documents are padded in the packed tensor (Megatron PackedSeqParams.cu_seqlens_q_padded).
   * Document z then occupies rows [cu_seqlens_padded[z], + cu_seqlens[z+1] - cu_seqlens[z]);
   * rows between documents are not read and not written. NULL: documents are contiguous. */
  const int32_t* cu_seqlens_padded;
  /* Backward only. 0: dq is accumulated across key blocks with fp32 reduce-adds in whatever order
   * the blocks finish, so it may differ in the last bits from run to run (dk, dv, dn, db are
   * always bit-reproducible). 1: the tensor-core backward adds every dQ tile's contributions in
   * ascending key-block order (bounded waits between CTAs; a wait that expires records
   * SSA_ERR_DEVICE_TIMEOUT), so dq is bit-identical from run to run, as the reference's
   * determinism suite requires (check_ssa_triton_parity.py:507-562). The generic kernels are
   * deterministic in both modes. Costs extra workspace and some speed. */
  int32_t deterministic;
  /* Output dropout, fused. The reference applies nn.Dropout(p) to the attention output after its
   * kernel, in training only (ssa_triton_attention.py:110-113,186-193). dropout_p in [0, 1);
   * 0 = off (dropout_seed is then not read). When > 0:
   *   - the forward writes out = O * keep / (1 - p), keep drawn per element from Philox4x32-10
   *     keyed by dropout_seed (device, two 64-bit values: [0] the key, [1] the counter offset;
   *     the element with logical index e, its position in contiguous [B, Hq, N, D] or packed
   *     [T, Hq, D], uses word e % 4 of the call with counter (e / 4, offset));
   *   - the backward takes that dropped `out` and the gradient of the dropped output as `dout`,
   *     with the same dropout_p and dropout_seed, and returns the gradients for
   *     dO = dout * keep / (1 - p): rowsum(out * dout) equals the undropped rowsum(O * dO); the
   *     kernels read dout * keep (written into the workspace: exact, no rounding of the scaled
   *     value) and apply 1 / (1 - p) in fp32 through delta and the normaliser.
   * lse is the undropped normaliser. ssa_attn_bwd_noalloc rejects dropout (no workspace for the
   * masked dout). */
  float dropout_p;
  const uint64_t* dropout_seed;
} ssa_problem_t;

/* Forward. Replaces ssa_flash_attn_forward (ssa_triton_kernel.py:732-792) and the
 * _ssa_attn_fwd launch (ssa_triton_kernel.py:776). Writes out (q's dtype) and lse. */
int ssa_attn_fwd(const ssa_problem_t* prob,
                 ssa_tensor_t q, ssa_tensor_t k, ssa_tensor_t v,
                 ssa_tensor_t out, float* lse,
                 void* workspace, size_t workspace_bytes, void* stream);
size_t ssa_attn_fwd_workspace_size(const ssa_problem_t* prob);

/* Backward preprocess: delta = rowsum(out * dout) in fp32, [B, Hq, N] contiguous.
 * Replaces _ssa_attn_bwd_preprocess (ssa_triton_kernel.py:267-298, launched at :832). */
int ssa_attn_bwd_preprocess(const ssa_problem_t* prob, ssa_tensor_t out, ssa_tensor_t dout,
                            float* delta, void* stream);

/* Backward. Replaces ssa_flash_attn_backward (ssa_triton_kernel.py:795-897): the
 * preprocess launch (:832), the fused _ssa_attn_bwd launch (:861) and the dn/db sums
 * (:894-895). Writes dq, dk, dv (q's dtype), dn (1 or Hq floats, device) and db (1 float,
 * device). dn/db are reduced on the device in fp64, deterministically. */
int ssa_attn_bwd(const ssa_problem_t* prob,
                 ssa_tensor_t q, ssa_tensor_t k, ssa_tensor_t v,
                 ssa_tensor_t out, ssa_tensor_t dout, const float* lse,
                 ssa_tensor_t dq, ssa_tensor_t dk, ssa_tensor_t dv,
                 float* dn, float* db,
                 void* workspace, size_t workspace_bytes, void* stream);
size_t ssa_attn_bwd_workspace_size(const ssa_problem_t* prob);

/* Backward that allocates nothing and takes no workspace. No counterpart in the reference.
 * For callers that cannot allocate device memory where they run the backward (a binding from
 * another host language with no device allocator, or a loop whose device memory is reserved
 * up front by another allocator). Runs the generic CUDA-core backward kernels with their
 * scratch (delta and dn/db partials) in a fixed 16 MiB device array owned by the library:
 * problems needing more return SSA_ERR_WORKSPACE; calls that overlap on one GPU race on the
 * array; the first call on each device resolves the array's address (make it before any stream
 * capture starts). Results match ssa_attn_bwd within the library's parity tolerances. */
int ssa_attn_bwd_noalloc(const ssa_problem_t* prob,
                         ssa_tensor_t q, ssa_tensor_t k, ssa_tensor_t v,
                         ssa_tensor_t out, ssa_tensor_t dout, const float* lse,
                         ssa_tensor_t dq, ssa_tensor_t dk, ssa_tensor_t dv,
                         float* dn, float* db, void* stream);

/* Which kernel family serves this problem: 0 = generic (fp32-compute SIMT: fp32 inputs or
 * D = 16, which has no tensor-core kernel), 1 = sm_100a tcgen05/TMA kernels (bf16/fp16 with
 * D in {32, 64, 128}; D = 32 runs the D = 64 kernels). */
int ssa_attn_kernel_family(const ssa_problem_t* prob);

/* Reads and clears the device status word written by bounded device-side waits
 * (synchronises `stream`). 0 = no error, else SSA_ERR_DEVICE_TIMEOUT. */
int ssa_device_status(void* stream);

/* Failure-path self-test: launches one kernel that waits on an mbarrier no thread completes,
 * through the same bounded wait the attention kernels use but limited to wait_cycles; the
 * expired wait records SSA_ERR_DEVICE_TIMEOUT in the device status word (read and clear it
 * with ssa_device_status; until then the attention kernels skip their work). No fault, no
 * trap. No reference counterpart. */
int ssa_selftest_device_timeout(uint64_t wait_cycles, void* stream);

/* Number of CUDA kernels this library has launched in this process (all devices, all
 * threads). Lets a caller count the device work behind a call without a profiler. */
uint64_t ssa_kernel_launch_count(void);

/* Human-readable description of the last error on this host thread. */
const char* ssa_last_error(void);

/* Library version string. */
const char* ssa_version(void);

#ifdef __cplusplus
}
#endif
#endif /* SSA_B200_H */

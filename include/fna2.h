/*
 * fna2.h -- C ABI of the B200-native (sm_100a) FNA2 fused relational-bias
 * attention library (libfna2_b200.so).
 *
 * Computes, per query head h, query row i and key row j of one sequence:
 *   S[i,j] = softmax_scale * <Q[i],K[j]> + gs[h] * <R_q[i],R_k[j]>   (h <  H_G)
 *   S[i,j] = softmax_scale * <Q[i],K[j]>                             (h >= H_G)
 *   S[i,j] = -inf when causal and j > i (positions local to the sequence)
 *   O = softmax(S) V,  O = acc/(l+1e-6),  LSE = m + log(l+1e-6)
 * with GQA kv_head = h / (H/H_KV), and the backward producing dQ, dK, dV,
 * dR_q, dR_k and d_graph_scale.
 *
 * The entry points replace the launchers of the reference Python/Triton
 * implementation (myAiByMe/FNA2, file FNA2/flash_naylis_attn.py):
 *   fna2_fwd  <- _fna2_forward        (flash_naylis_attn.py:700-753)
 *                _fna2_forward_varlen (flash_naylis_attn.py:756-804)
 *   fna2_bwd  <- _fna2_backward        (flash_naylis_attn.py:807-892)
 *                _fna2_backward_varlen (flash_naylis_attn.py:1215-1300)
 * The reference's public op flash_naylis_attn() (flash_naylis_attn.py:1380)
 * and its autograd Function (:1307-1373) are mirrored in Python by
 * fna2_b200/flash_naylis_attn.py on top of these calls.
 *
 * Conventions
 *   - All tensor pointers are device pointers; q/k/v/out/dout/r_q/r_k and all
 *     gradients except d_graph_scale are bf16; graph_scale, lse and
 *     d_graph_scale are fp32; cu_seqlens are int32.
 *   - Fna2Tensor.stride holds element strides for (batch, head, row, col).
 *     Dense tensors are [B, heads, S, X]; packed (varlen) tensors are
 *     [T, heads, X] and use stride[0] = 0 (ignored), stride[1] = head stride,
 *     stride[2] = token stride.  The column stride must be 1; the other
 *     strides and every base pointer must be 16-byte aligned (TMA rule).
 *   - lse is fp32, contiguous: [B, H, S] for dense problems and [H, T_q] for
 *     packed ones.
 *   - Varlen problems are always causal (the reference's varlen kernel has no
 *     is_causal argument, flash_naylis_attn.py:1327-1332).
 *   - Work is enqueued on `stream` (a cudaStream_t, NULL = legacy default);
 *     the calls never synchronise the host.
 *   - Return value: 0 on success, FNA2_ERR_INVALID (-1) for bad arguments
 *     (message in fna2_last_error()), FNA2_ERR_CUDA (-2) when a CUDA call
 *     failed (message likewise), FNA2_ERR_WORKSPACE (-3) for a too small
 *     workspace.
 */
#ifndef FNA2_B200_H_
#define FNA2_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FNA2_ABI_VERSION 5

#define FNA2_OK 0
#define FNA2_ERR_INVALID (-1)
#define FNA2_ERR_CUDA (-2)
#define FNA2_ERR_WORKSPACE (-3)

typedef struct Fna2Tensor {
  void* ptr;         /* device pointer (NULL allowed only where noted) */
  int64_t stride[4]; /* element strides: batch, head, row, col */
} Fna2Tensor;

typedef struct Fna2Problem {
  int32_t batch;       /* dense: B.  varlen: number of packed sequences N */
  int32_t seqlen_q;    /* dense: S.  varlen: max_seqlen_q (>= every q length) */
  int32_t seqlen_k;    /* dense: S.  varlen: max_seqlen_k (>= every k length) */
  int32_t total_q;     /* varlen: rows of the packed q tensor (T_q); dense: unused */
  int32_t total_k;     /* varlen: rows of the packed k/v tensors (T_k); dense: unused */
  int32_t heads;       /* H */
  int32_t heads_kv;    /* H_KV, divides H */
  int32_t heads_graph; /* H_G <= H: heads [0, H_G) carry the rank-r bias */
  int32_t head_dim;    /* D: 64 or 128 */
  int32_t rank;        /* r: multiple of 8, <= 32 (ignored when H_G == 0) */
  float softmax_scale; /* the reference defaults it to 1/sqrt(D) (:1415-1416) */
  int32_t causal;      /* dense only; varlen is always causal */
  const int32_t* cu_seqlens_q; /* varlen: device [N+1] cumulative q lengths; dense: NULL */
  const int32_t* cu_seqlens_k; /* varlen: device [N+1] cumulative k lengths; dense: NULL */
} Fna2Problem;

typedef struct Fna2FwdArgs {
  Fna2Problem prob;
  Fna2Tensor q, k, v;   /* [B,H,S,D] / [B,H_KV,S,D]  or  [T,H,D] / [T,H_KV,D] */
  Fna2Tensor r_q, r_k;  /* [B,H_G,S,r] or [T,H_G,r] (ptr may be NULL if H_G == 0) */
  const float* graph_scale; /* [H_G] */
  Fna2Tensor out;       /* same shape as q */
  float* lse;           /* [B,H,S] or [H,T_q] */
  void** launch_events; /* optional (NULL = off): 2 cudaEvent_t recorded on `stream`
                           before and after the forward (for packed batches: the tile
                           table kernel and the forward kernel), for per-kernel timing */
  void* workspace;      /* packed batches: device scratch, >= fna2_fwd_workspace_size()
                           bytes, 256-B aligned (the table of real query-tile pairs:
                           32 B per entry, ceil(T_q/256) + N entries); dense: unused */
  size_t workspace_bytes;
} Fna2FwdArgs;

typedef struct Fna2BwdArgs {
  Fna2Problem prob;
  Fna2Tensor q, k, v, r_q, r_k;
  const float* graph_scale;
  Fna2Tensor out, dout;      /* forward output and upstream gradient (shape of q) */
  const float* lse;          /* as written by fna2_fwd */
  Fna2Tensor dq, dk, dv, dr_q, dr_k; /* outputs, shapes of the inputs */
  float* d_graph_scale;      /* [H_G] output (overwritten) */
  void* workspace;           /* device scratch, >= fna2_bwd_workspace_size() bytes, 256-B aligned */
  size_t workspace_bytes;
  void** launch_events;      /* optional (NULL = off): 4 cudaEvent_t recorded on `stream` before the
                                pre-pass, after it, after the dK/dV kernel and after the dQ kernel */
} Fna2BwdArgs;

/* Bytes of device scratch fna2_fwd needs for this problem (0 for dense
 * problems or if invalid).  The reference's forward launcher allocates none: its
 * varlen grid is (tiles of max_seqlen) x heads x sequences (flash_naylis_attn.py:
 * 786-793); this one launches one CTA per real pair of query tiles from the table. */
size_t fna2_fwd_workspace_size(const Fna2Problem* prob);

/* Forward: writes out and lse.  Replaces _fna2_forward / _fna2_forward_varlen. */
int fna2_fwd(const Fna2FwdArgs* args, void* stream);

/* Bytes of device scratch fna2_bwd needs for this problem (0 if invalid). */
size_t fna2_bwd_workspace_size(const Fna2Problem* prob);

/* Backward: writes dq, dk, dv, dr_q, dr_k and d_graph_scale.
 * Replaces _fna2_backward / _fna2_backward_varlen. */
int fna2_bwd(const Fna2BwdArgs* args, void* stream);

/* Size of the device scratch array behind fna2_bwd_noalloc (32 MiB per GPU). */
#define FNA2_NOALLOC_SCRATCH_BYTES (32 * 1024 * 1024)

/* Backward for callers that cannot allocate device memory (no counterpart in
 * the reference, which always allocates through PyTorch).  Same arguments and
 * results as fna2_bwd, but args->workspace / workspace_bytes are ignored: the
 * scratch (8 bytes per query row and head, plus 32 bytes per 128-row query
 * tile and per 128-row key tile of packed batches) comes from a static device array of
 * FNA2_NOALLOC_SCRATCH_BYTES held by every GPU that loads the library until
 * exit.  Larger problems return FNA2_ERR_WORKSPACE.  The first call on each
 * device looks the array up (cudaGetSymbolAddress); make it before any stream
 * capture.  All calls on a device share the array: calls whose GPU work
 * overlaps race on it, so order them on one stream.  Calls no cudaMalloc or
 * cudaFree. */
int fna2_bwd_noalloc(const Fna2BwdArgs* args, void* stream);

/* ------------------------------------------------------------------------
 * Varlen QK-RMSNorm + RoPE: the transform NaylisAttention._forward_varlen
 * applies to q and k before the attention (FNA2/attention_fna2.py:558-566:
 * RMSNorm :94-102, RotaryPositionalEmbedding :108-163, _apply_rope_varlen
 * :620-647), fused into one pass whose positions restart at 0 for every
 * packed sequence (the reference loops over sequences on the host after a
 * .tolist() sync).  Per row x (one token, one head, head_dim values):
 *   n = x * rsqrt(mean(x^2) + eps) * w                 (if the weight is set)
 *   y = n * cos(pos * f) + rotate_half(n) * sin(pos * f) (if inv_freq is set)
 * with f = inv_freq repeated twice over head_dim, pos the token's index
 * within its sequence, rotate_half(n) = [-n[D/2:], n[:D/2]], and y stored
 * as bf16 (the attention's input dtype).  The cos/sin table is formed in
 * rope_dtype as the reference does (in bf16, positions and angles are
 * rounded to bf16 first).  Tokens outside [cu[0], cu[N]) are not written by
 * the forward when RoPE is on (the reference leaves them unset) and get zero
 * gradients.  head_dim is 64 or 128.
 * Replace: RMSNorm.forward (attention_fna2.py:100-102) on q and k, and
 * NaylisAttention._apply_rope_varlen (:620-647). */
#define FNA2_DTYPE_F32 0
#define FNA2_DTYPE_BF16 1

typedef struct Fna2Rows { /* [T, heads, head_dim] rows, column stride 1 */
  void* ptr;
  int64_t token_stride; /* elements */
  int64_t head_stride;  /* elements */
} Fna2Rows;

typedef struct Fna2QkPrepArgs {
  int64_t total_tokens;       /* T */
  int num_seqs;               /* N */
  const int32_t* cu_seqlens;  /* [N+1], device */
  int heads_q, heads_k, head_dim;
  int in_dtype;               /* dtype of q_in and k_in (FNA2_DTYPE_*) */
  int weight_dtype;           /* dtype of q_weight and k_weight */
  int rope_dtype;             /* dtype of the tensor entering RoPE in the reference */
  Fna2Rows q_in, k_in;
  Fna2Rows q_out, k_out;      /* bf16 */
  const void* q_weight;       /* [head_dim] RMSNorm weight, or NULL: no norm */
  const void* k_weight;
  float eps;
  const float* inv_freq;      /* [head_dim/2] fp32, or NULL: no RoPE */
} Fna2QkPrepArgs;

/* Forward of the transform above. */
int fna2_qk_prep_fwd(const Fna2QkPrepArgs* args, void* stream);

typedef struct Fna2QkPrepBwdArgs {
  Fna2QkPrepArgs fwd;         /* the forward's arguments; q_in/k_in are read again, q_out/k_out unused */
  Fna2Rows dq_out, dk_out;    /* gradients of the bf16 outputs (bf16) */
  Fna2Rows dq_in, dk_in;      /* written, in in_dtype */
  float* dq_weight;           /* [head_dim] fp32, accumulated into (zero it first), or NULL */
  float* dk_weight;
} Fna2QkPrepBwdArgs;

/* Backward of the transform: gradients of q_in, k_in and of the two weights. */
int fna2_qk_prep_bwd(const Fna2QkPrepBwdArgs* args, void* stream);

/* ---------------------------------------------------------------------------
 * KV-cache decode with the relational bias.  No counterpart in the reference:
 * its decode step (attention_fna2.py:428-432, past_kv set) bypasses FNA2 and
 * drops graph_bias because R_k is not cached.  Here R_k is cached per graph
 * head next to K and V, and one new query token per sequence attends to keys
 * [0, cache_seqlens[b]) of its sequence -- plus its own new key when k_new is
 * given, which the call also writes into the caches at slot cache_seqlens[b]
 * (the caller then advances cache_seqlens).  Logits are those of the last
 * query row of the prefill op above (no causal mask is needed: the query
 * sits after every key), and out/lse follow its normalisation.
 *
 * Layouts (element strides; column stride 1; bases and strides 16-byte
 * aligned): q [B, H, D], r_q [B, H_G, R], out [B, H, D]; caches
 * k/v [B, capacity, H_KV, D] and r_k [B, capacity, H_G, R] addressed as
 * base + b*batch_stride + slot*token_stride + head*head_stride, or, when
 * cache_offsets is set, base + (cache_offsets[b] + slot)*token_stride +
 * head*head_stride (packed caches; batch strides ignored); k_new/v_new
 * [B, H_KV, D], rk_new [B, H_G, R].  lse (optional) is fp32 [B, H].
 * A sequence with cache_seqlens[b] < 0 or more keys than capacity makes the
 * kernel record site code 601 (fna2_device_status) and write zeros.
 * --------------------------------------------------------------------------- */
typedef struct Fna2DecodeArgs {
  int batch, heads, kv_heads, graph_heads, head_dim, rank;
  int capacity;                 /* cache slots per sequence */
  float softmax_scale;
  const void* q;        int64_t q_batch_stride, q_head_stride;
  const void* r_q;      int64_t rq_batch_stride, rq_head_stride;
  void* k_cache;        int64_t k_batch_stride, k_token_stride, k_head_stride;
  void* v_cache;        int64_t v_batch_stride, v_token_stride, v_head_stride;
  void* rk_cache;       int64_t rk_batch_stride, rk_token_stride, rk_head_stride;
  const float* graph_scale;     /* [H_G] */
  const int32_t* cache_seqlens; /* [B], device */
  const int32_t* cache_offsets; /* [B], device, or NULL */
  const void* k_new;    int64_t kn_batch_stride, kn_head_stride;  /* or NULL (then v_new, rk_new too) */
  const void* v_new;    int64_t vn_batch_stride, vn_head_stride;
  const void* rk_new;   int64_t rkn_batch_stride, rkn_head_stride;
  void* out;            int64_t out_batch_stride, out_head_stride;
  float* lse;                   /* or NULL */
  int num_splits;               /* key splits per (sequence, head); 0 = chosen by the library */
} Fna2DecodeArgs;

/* Bytes of fp32 workspace fna2_decode needs for these arguments (0 when the
 * keys of a (sequence, head) are not split). */
size_t fna2_decode_workspace_size(const Fna2DecodeArgs* args);

int fna2_decode(const Fna2DecodeArgs* args, void* workspace, size_t workspace_bytes, void* stream);

/* Message of the last failed call on this host thread ("" if none). */
const char* fna2_last_error(void);

/* Device status: returns the first site code a kernel recorded since the last
 * reset (0 = none) and clears it when reset != 0.  Synchronises the current
 * device.  Codes:
 *   1xx-10xx  a bounded mbarrier wait gave up after its budget (4 s): the
 *             kernel raised its CTA's abort flag, skipped the rest of the
 *             tile and deallocated its tensor memory (hundreds digit = kernel
 *             role: 1-3 forward, 4-7 dK/dV, 8-10 dQ);
 *   199, 499  the dynamic shared memory base was not 1024-byte aligned;
 *   601       decode: a cache length < 0 or above the capacity (zeros written);
 *   621       forward, packed batch: a sequence with inconsistent cu_seqlens
 *             (negative length, rows outside [0, total_q/total_k), or longer
 *             than max_seqlen_q/_k); the sequence is skipped, its out/lse rows
 *             are not written;
 *   622       backward pre-pass, packed batch: the same check; the sequence
 *             gets no tiles and its gradient rows are not written.
 * Neither the reference nor this library checks cu_seqlens on the host (that
 * would need a device-to-host copy per call). */
int fna2_device_status(int reset);

/* Testing hook (no counterpart in the reference): makes the forward kernel
 * withhold one mbarrier arrival (withhold_site = 204: the first P hand-off of
 * each CTA's first query tile) and sets the wait budget to wait_limit_ns
 * (0 = the default 4 s), so that a test can check that a wait which runs out
 * records its site code, that the kernel exits cleanly and that the next call
 * works.  fna2_debug_watchdog(0, 0) restores normal operation.  Synchronises
 * the current device. */
int fna2_debug_watchdog(int withhold_site, unsigned long long wait_limit_ns);

/* Dense bf16 GEMM for the stacked R_q / R_k projection (replaces the two
 * nn.Linear layers rel_q_proj / rel_k_proj of FNA2/attention_fna2.py:320-335
 * and the products autograd forms for them):
 *   c_dtype == FNA2_DTYPE_BF16:  C[m][n]  = sum_k A[m][k] B[n][k]   (stored)
 *   c_dtype == FNA2_DTYPE_F32:   C[m][n] += sum_k A[m][k] B[n][k]   (added; K may be
 *                                split into split_k slices reduced with fp32 atomics;
 *                                C is not cleared)
 * A is bf16, K-major (A[m][k] at a[m*lda + k]) or, with a_mn_major = 1,
 * M-major (A[m][k] at a[k*lda + m]); B likewise with N.  fp32 accumulation.
 * Requirements: m, n, k >= 1; n a multiple of 32; 16-byte aligned a, b, c;
 * lda, ldb multiples of 8 elements and ldc of 8 (bf16) or 4 (fp32) elements;
 * split_k >= 1, and 1 for bf16 output.  FNA2_ERR_INVALID otherwise. */
typedef struct Fna2GemmArgs {
  int64_t m, n, k;
  const void* a;
  int64_t lda;
  int32_t a_mn_major;
  const void* b;
  int64_t ldb;
  int32_t b_mn_major;
  void* c;
  int64_t ldc;
  int32_t c_dtype;
  int32_t split_k;
} Fna2GemmArgs;
int fna2_gemm(const Fna2GemmArgs* args, void* stream);

/* FNA2_ABI_VERSION of the loaded library. */
int fna2_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FNA2_B200_H_ */

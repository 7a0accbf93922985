// Device-side parameter blocks and shared constants of the FNA2 kernels.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>

namespace fna2 {

constexpr int kMaxDynamicSmem = 232448;  // 227 KB: dynamic shared memory per block on sm_100
constexpr int kBlockM = 128;  // query rows per tile (one TMEM lane / softmax thread per row)
constexpr int kBlockN = 128;  // key rows per tile
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kEps = 1e-6f;  // O = acc/(l+1e-6), LSE = m + log(l+1e-6)  (flash_naylis_attn.py:192,195)

// Query rows per tile of the key-stationary backward kernel: the largest of
// 96, 80 and 64 for which dV, [dK | dR_k], S^T, dP^T and a separate packed P^T
// fit in the 512 TMEM columns (D + D + r_pad + 2.5 QT <= 512); the two
// softmax warpgroups take 48 + 48, 48 + 32 or 32 + 32 query columns.
__host__ __device__ constexpr int dkdv_query_rows(int D, int RP) { return (D == 128 && RP == 32) ? 80 : 96; }

// Key rows per tile of the query-stationary (dQ) backward kernel: [dQ | dR_q]
// (160 columns), S and dP (112 each; dS is written over dP's first columns),
// Q and dO (64 each) fill the 512 TMEM columns.
__host__ __device__ constexpr int dq_key_rows(int /*D*/, int /*RP*/) { return 112; }

// Sequence bounds of one (batch or packed sequence) index. Dense problems have
// all sequences of length seqlen_q/seqlen_k starting at row 0 of their batch.
struct SeqInfo {
  int q_start, k_start;  // first row in the row dimension of the tensor maps
  int len_q, len_k;      // sequence lengths
  int b;                 // batch coordinate (0 for varlen)
};

struct ProblemDev {
  int heads, heads_kv, heads_graph, head_dim, rank;
  int seqlen_q, seqlen_k;  // dense lengths; varlen: max lengths (grid sizing only)
  int total_q, total_k;    // varlen: rows of the packed q and k/v tensors
  int varlen, causal;
  // varlen grids: 0 = (table entry, head), 1 = (head, table entry); see head_fast_grid
  int head_fast;
  const int* cu_q;
  const int* cu_k;
  float scale;       // softmax_scale
  float scale_log2;  // softmax_scale * log2(e)
  const float* gs;   // graph_scale [H_G]
};

// Grid coordinates of a varlen kernel launched over (table entry, head): the
// entry is the fast dimension unless p.head_fast (small problems), in which
// case every head's heaviest tiles are dispatched before any lighter ones.
__device__ __forceinline__ int grid_entry(const ProblemDev& p) { return p.head_fast ? blockIdx.y : blockIdx.x; }
__device__ __forceinline__ int grid_head(const ProblemDev& p) {
  return (p.varlen && p.head_fast) ? blockIdx.x : blockIdx.y;
}

__device__ __forceinline__ SeqInfo seq_info(const ProblemDev& p, int bz) {
  SeqInfo s;
  if (p.varlen) {
    s.q_start = __ldg(p.cu_q + bz);
    s.len_q = __ldg(p.cu_q + bz + 1) - s.q_start;
    s.k_start = __ldg(p.cu_k + bz);
    s.len_k = __ldg(p.cu_k + bz + 1) - s.k_start;
    s.b = 0;
  } else {
    s.q_start = 0;
    s.k_start = 0;
    s.len_q = p.seqlen_q;
    s.len_k = p.seqlen_k;
    s.b = bz;
  }
  return s;
}

// Site codes a kernel records in g_device_error (read by fna2_device_status)
// when a packed sequence's cu_seqlens entries are inconsistent: a negative
// length, rows outside the packed tensors, or a length above max_seqlen (the
// bound the grids are sized by).  The sequence is skipped before any access.
constexpr int kStatusBadSeqFwd = 621;  // found by the forward kernel
constexpr int kStatusBadSeqBwd = 622;  // found by the backward pre-pass (tile tables)

// A packed sequence the kernels may process: inside the packed tensors and no
// longer than the max_seqlen bounds.  Dense problems always pass.
__device__ __forceinline__ bool seq_ok(const ProblemDev& p, const SeqInfo& s) {
  if (!p.varlen) return true;
  const int64_t qe = static_cast<int64_t>(s.q_start) + s.len_q, ke = static_cast<int64_t>(s.k_start) + s.len_k;
  return s.q_start >= 0 && s.len_q >= 0 && qe <= p.total_q && s.len_q <= p.seqlen_q && s.k_start >= 0 &&
         s.len_k >= 0 && ke <= p.total_k && s.len_k <= p.seqlen_k;
}

struct FwdParams {
  ProblemDev prob;
  __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_sr;  // element strides (batch, head, row); column stride is 1
  float* lse;                // index (b*H + h) * lse_sbh + row
  int64_t lse_sbh;
  int n_mblocks;             // dense: query tiles per sequence (grid.x = pairs of them)
  // varlen: table of the real pairs of 128-row query tiles, 8 ints per entry
  // {pair, q_start, k_start, len_q, len_k, 0, 0, 0} (pair < 0: past the end),
  // written by fna2_fwd_table_kernel; the forward launches tab_len CTAs per head
  int4* tab;
  int tab_len;
};

struct BwdParams {
  ProblemDev prob;
  // forward output / upstream gradient, row-major bf16 with unit column stride
  const __nv_bfloat16* out;
  int64_t o_sb, o_sh, o_sr;
  const __nv_bfloat16* dout;
  int64_t do_sb, do_sh, do_sr;
  const __nv_bfloat16* q;  // read row-wise into tensor memory by the query-stationary kernel
  int64_t q_sb, q_sh, q_sr;
  const float* lse;  // forward LSE, index (b*H + h) * lse_sbh + row
  int64_t lse_sbh;
  // workspace: per (b*H + h) rows of log2-domain LSE and Delta = rowsum(dO*O)
  float* ws_lse2;
  float* ws_delta;
  int64_t ws_sbh;  // rows per (b,h) slot in the workspace (>= rows of the q tensor)
  // gradients
  __nv_bfloat16* dq;
  int64_t dq_sb, dq_sh, dq_sr;
  __nv_bfloat16* dk;
  int64_t dk_sb, dk_sh, dk_sr;
  __nv_bfloat16* dv;
  int64_t dv_sb, dv_sh, dv_sr;
  __nv_bfloat16* drq;
  int64_t drq_sb, drq_sh, drq_sr;
  __nv_bfloat16* drk;
  int64_t drk_sb, drk_sh, drk_sr;
  const __nv_bfloat16* rq;  // raw R_q rows (for d_gs = sum R_q * dS R_k)
  int64_t rq_sb, rq_sh, rq_sr;
  float* dgs;               // [H_G], accumulated with atomics (zeroed by the pre kernel)
  // varlen: tables of the real tiles, 8 ints per entry {tile, q_start, k_start, len_q,
  // len_k, 0, 0, 0} (tile < 0: past the end), written by the pre kernel; the dQ kernel
  // launches tab_q_len CTAs per head (query tiles), the dK/dV kernel tab_k_len (key tiles)
  int4* tab_q;
  int4* tab_k;
  int tab_q_len, tab_k_len;
  int total_q_rows;         // rows of q per (b,h) slot: dense S, varlen T
  int total_k_rows;
  int batch;                // dense B or varlen N
  int n_mblocks, n_nblocks;
};

// Tensor maps of one backward call.  Each kernel tiles its stationary operand
// by 128 rows and streams the other in smaller tiles; the streamed R operand
// is read as a zero-padded 64-column swizzle atom next to Q (dK/dV) or K (dQ).
struct BwdMaps {
  CUtensorMap q, k, v, dO, rq, rk;  // 128-row boxes (R with r_pad-column boxes)
  CUtensorMap qS, dOS, rqS;         // dkdv_query_rows-row boxes, streamed by the key-stationary kernel
  CUtensorMap kDq, vDq, rkDq;       // dq_key_rows-row boxes, streamed by the query-stationary kernel
};

}  // namespace fna2

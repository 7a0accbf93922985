// FNA2 backward on sm_100a.
//
// Reference semantics: FNA2/flash_naylis_attn.py:356-693 (dense) and
// :900-1208 (varlen): Delta = rowsum(dO*O) (:381), P = exp(S - LSE) (:518),
// dS = P*(dP - Delta) (:523), dV = P^T dO (:527), dK = scale*dS^T Q (:529),
// dR_k = gs*dS^T R_q (:535), dQ = scale*dS K (:679), dR_q = gs*dS R_k (:683),
// d_gs[h] = sum(dS * R_q R_k^T) (:537-538).  d_gs is formed here from the
// identity d_gs[h] = sum_i <R_q[i], (dS R_k)[i]>, so R_q R_k^T is never
// recomputed for it.
//
// Three launches:
//   fna2_bwd_pre_kernel   Delta and the LSE in log2 units into the workspace;
//                         zeroes d_gs and (varlen) gradient rows that belong
//                         to no sequence, as the reference's zeros_like does.
//   fna2_bwd_dkdv_kernel  one CTA per (128-row key tile, KV head, sequence),
//                         looping over the query heads of the GQA group and
//                         the causally visible query tiles.  TMEM: dV and
//                         [dK | dR_k] accumulators; S^T = K Q^T + R~_k R_q^T
//                         and dP^T = V dO^T per step; the softmax warps write
//                         P^T and dS^T back into TMEM as bf16 and the TS-form
//                         MMAs dV += P^T dO, [dK | dR_k] += dS^T [Q | R_q]
//                         read them from there.  No dK/dV atomics.
//   fna2_bwd_dq_kernel    one CTA per (128-row query tile, head, sequence),
//                         looping over the causally visible key tiles:
//                         S, dP, dS (bf16 into TMEM), dQ += dS K and
//                         dR_q += dS R_k (TS-form), then d_gs via one atomic
//                         per warp.
// The rank-r bias is one extra K-slice (K = r_pad) of each score MMA, with one
// side pre-scaled by gs/scale in shared memory (R~_k in the dK/dV kernel, R~_q
// in the dQ kernel).
#include <type_traits>

#include "fna2_kernels.cuh"
#include "ptx.cuh"

namespace fna2 {

inline size_t bwd_ws_align(size_t x) { return (x + 255) & ~size_t(255); }

// Varlen tile tables: at most ceil(T/128) + N real tiles per kind (query tiles for
// the dQ kernel, key tiles for the dK/dV kernel), 32 bytes per entry.
inline int bwd_tab_len(int rows, int n_seqs) { return (rows + kBlockM - 1) / kBlockM + n_seqs; }

// Workspace: log2-domain LSE and Delta (fp32 per query row and head), then, for
// varlen problems, the two tile tables.
inline size_t bwd_workspace_bytes(int batch_dim, int H, int /*HG*/, int rows, bool varlen = false, int rows_k = 0,
                                  int n_seqs = 0) {
  const size_t n = static_cast<size_t>(batch_dim) * H * rows;
  size_t bytes = 2 * bwd_ws_align(n * sizeof(float));
  if (varlen)
    bytes += bwd_ws_align((static_cast<size_t>(bwd_tab_len(rows, n_seqs)) + bwd_tab_len(rows_k, n_seqs)) * 32);
  return bytes;
}

inline void bwd_set_workspace(BwdParams* p, void* ws, int batch_dim, int H, int rows, bool varlen = false,
                              int rows_k = 0, int n_seqs = 0) {
  const size_t n = static_cast<size_t>(batch_dim) * H * rows;
  p->ws_lse2 = static_cast<float*>(ws);
  p->ws_delta = reinterpret_cast<float*>(static_cast<char*>(ws) + bwd_ws_align(n * sizeof(float)));
  p->ws_sbh = rows;
  p->tab_q = p->tab_k = nullptr;
  p->tab_q_len = p->tab_k_len = 0;
  if (varlen) {
    p->tab_q_len = bwd_tab_len(rows, n_seqs);
    p->tab_k_len = bwd_tab_len(rows_k, n_seqs);
    p->tab_q = reinterpret_cast<int4*>(static_cast<char*>(ws) + 2 * bwd_ws_align(n * sizeof(float)));
    p->tab_k = p->tab_q + 2 * static_cast<size_t>(p->tab_q_len);
  }
}

__device__ __forceinline__ void zero_row(__nv_bfloat16* row, int n) {
  uint4 z = make_uint4(0, 0, 0, 0);
  for (int c = 0; c < n; c += 8) *reinterpret_cast<uint4*>(row + c) = z;
}

// ---------------------------------------------------------------------------
// pre-pass: Delta = rowsum(dO*O), lse2 = LSE*log2(e)
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(128) fna2_bwd_pre_kernel(const BwdParams p) {
  const ProblemDev& P = p.prob;
  const int h = blockIdx.y;
  const int bz = blockIdx.z;
  const int row = blockIdx.x * 128 + threadIdx.x;
  if (blockIdx.x == 0 && h == 0 && bz == 0 && p.dgs != nullptr && static_cast<int>(threadIdx.x) < P.heads_graph)
    p.dgs[threadIdx.x] = 0.f;
  if (blockIdx.x == 0 && h == 0 && bz == 0 && P.varlen) {
    // tile tables of the varlen kernels: per sequence (in order) its query tiles, heaviest
    // causal tile first, and its key tiles; the unused tail is marked with tile = -1
    __shared__ int scan_s[2][4];
    int carry_q = 0, carry_k = 0;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    for (int base = 0; base < p.batch; base += 128) {
      const int z = base + static_cast<int>(threadIdx.x);
      int qs = 0, ks = 0, lq = 0, lk = 0;
      if (z < p.batch) {
        SeqInfo e;
        e.q_start = __ldg(P.cu_q + z), e.len_q = __ldg(P.cu_q + z + 1) - e.q_start;
        e.k_start = __ldg(P.cu_k + z), e.len_k = __ldg(P.cu_k + z + 1) - e.k_start;
        if (seq_ok(P, e)) {
          qs = e.q_start, lq = e.len_q, ks = e.k_start, lk = e.len_k;
        } else {  // inconsistent cu_seqlens: the sequence gets no tiles (no access is made for it)
          atomicCAS(&g_device_error, 0, kStatusBadSeqBwd);
        }
      }
      // lq, lk >= 0 here, so every table offset below stays in [0, tab_len)
      const int tq = (lq + kBlockM - 1) / kBlockM, tk = (lk + kBlockN - 1) / kBlockN;
      int iq = tq, ik = tk;  // inclusive scans within the warp
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int uq = __shfl_up_sync(0xffffffffu, iq, o), uk = __shfl_up_sync(0xffffffffu, ik, o);
        if (lane >= o) iq += uq, ik += uk;
      }
      if (lane == 31) scan_s[0][w] = iq, scan_s[1][w] = ik;
      __syncthreads();
      int oq = carry_q + iq - tq, ok = carry_k + ik - tk;
      for (int i = 0; i < w; ++i) oq += scan_s[0][i], ok += scan_s[1][i];
      for (int t = 0; t < tq && oq + t < p.tab_q_len; ++t) {
        p.tab_q[2 * (oq + t)] = make_int4(tq - 1 - t, qs, ks, lq);
        p.tab_q[2 * (oq + t) + 1] = make_int4(lk, z, 0, 0);
      }
      for (int t = 0; t < tk && ok + t < p.tab_k_len; ++t) {
        p.tab_k[2 * (ok + t)] = make_int4(t, qs, ks, lq);
        p.tab_k[2 * (ok + t) + 1] = make_int4(lk, z, 0, 0);
      }
      carry_q += scan_s[0][0] + scan_s[0][1] + scan_s[0][2] + scan_s[0][3];
      carry_k += scan_s[1][0] + scan_s[1][1] + scan_s[1][2] + scan_s[1][3];
      __syncthreads();
    }
    for (int i = carry_q + static_cast<int>(threadIdx.x); i < p.tab_q_len; i += 128)
      p.tab_q[2 * i] = make_int4(-1, 0, 0, 0);
    for (int i = carry_k + static_cast<int>(threadIdx.x); i < p.tab_k_len; i += 128)
      p.tab_k[2 * i] = make_int4(-1, 0, 0, 0);
  }
  {
    // Delta = rowsum(dO * O): a row is read by D/8 lanes (16 bytes each), so every
    // load instruction covers whole rows; each warp owns 32 of the block's rows.
    constexpr int LPR = D / 8, RPI = 32 / LPR, ITERS = 32 / RPI, BATCH = ITERS < 8 ? ITERS : 8;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane % LPR, rsel = lane / LPR;
    const int row_base = blockIdx.x * 128 + warp * 32;
    const int64_t sbh = static_cast<int64_t>(bz) * P.heads + h;
#pragma unroll
    for (int i0 = 0; i0 < ITERS; i0 += BATCH) {
      uint4 a[BATCH], b[BATCH];
#pragma unroll
      for (int i = 0; i < BATCH; ++i) {
        const int r = row_base + (i0 + i) * RPI + rsel;
        a[i] = b[i] = make_uint4(0u, 0u, 0u, 0u);
        if (r < p.total_q_rows) {
          a[i] = *reinterpret_cast<const uint4*>(p.out + bz * p.o_sb + h * p.o_sh + static_cast<int64_t>(r) * p.o_sr +
                                                 sub * 8);
          b[i] = *reinterpret_cast<const uint4*>(p.dout + bz * p.do_sb + h * p.do_sh +
                                                 static_cast<int64_t>(r) * p.do_sr + sub * 8);
        }
      }
      float acc[BATCH];
#pragma unroll
      for (int i = 0; i < BATCH; ++i) {
        const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a[i]);
        const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&b[i]);
        acc[i] = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 x = __bfloat1622float2(a2[k]);
          const float2 y = __bfloat1622float2(b2[k]);
          acc[i] = fmaf(x.x, y.x, acc[i]);
          acc[i] = fmaf(x.y, y.y, acc[i]);
        }
      }
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1)
#pragma unroll
        for (int i = 0; i < BATCH; ++i) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
#pragma unroll
      for (int i = 0; i < BATCH; ++i) {
        const int r = row_base + (i0 + i) * RPI + rsel;
        if (sub == 0 && r < p.total_q_rows) {
          p.ws_delta[sbh * p.ws_sbh + r] = acc[i];
          p.ws_lse2[sbh * p.ws_sbh + r] = p.lse[sbh * p.lse_sbh + r] * kLog2e;
        }
      }
    }
  }
  if (P.varlen) {
    // rows outside [cu[0], cu[N]) are not owned by any tile: zero them
    const int q_lo = __ldg(P.cu_q), q_hi = __ldg(P.cu_q + p.batch);
    const int k_lo = __ldg(P.cu_k), k_hi = __ldg(P.cu_k + p.batch);
    if (row < p.total_q_rows && (row < q_lo || row >= q_hi)) {
      zero_row(p.dq + h * p.dq_sh + static_cast<int64_t>(row) * p.dq_sr, D);
      if (h < P.heads_graph) zero_row(p.drq + h * p.drq_sh + static_cast<int64_t>(row) * p.drq_sr, P.rank);
    }
    if (row < p.total_k_rows && (row < k_lo || row >= k_hi)) {
      if (h < P.heads_kv) {
        zero_row(p.dk + h * p.dk_sh + static_cast<int64_t>(row) * p.dk_sr, D);
        zero_row(p.dv + h * p.dv_sh + static_cast<int64_t>(row) * p.dv_sr, D);
      }
      if (h < P.heads_graph) zero_row(p.drk + h * p.drk_sh + static_cast<int64_t>(row) * p.drk_sr, P.rank);
    }
  }
}

// ---------------------------------------------------------------------------
// shared helpers
// ---------------------------------------------------------------------------
template <int RP>
__device__ __forceinline__ void scale_rows_inplace(uint8_t* base, int row, float f) {
  uint4* rrow = reinterpret_cast<uint4*>(base + row * RP * 2);
#pragma unroll
  for (int u = 0; u < RP / 8; ++u) {
    uint4 w = rrow[u];
    uint32_t* e = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f2 = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&e[i]));
      e[i] = pack_bf16(f2.x * f, f2.y * f);
    }
    rrow[u] = w;
  }
}

// Store 32 fp32 values (scaled) as bf16 to a row (16-byte aligned).
__device__ __forceinline__ void store_row32(__nv_bfloat16* dst, const uint32_t* v, float f) {
  uint4 w[4];
  uint32_t* wp = reinterpret_cast<uint32_t*>(w);
#pragma unroll
  for (int i = 0; i < 16; ++i) wp[i] = pack_bf16(__uint_as_float(v[2 * i]) * f, __uint_as_float(v[2 * i + 1]) * f);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) d4[i] = w[i];
}

__device__ __forceinline__ uint32_t r_layout_of(int rp) {
  return rp == 16 ? kSwizzle32B : (rp == 32 ? kSwizzle64B : kSwizzle128B);
}

// ---------------------------------------------------------------------------
// dK / dV / dR_k  (KV-stationary)
// ---------------------------------------------------------------------------
// One CTA per (128-row key tile, KV head, sequence), looping over the query
// heads of the GQA group and the causally visible query tiles of QT rows
// (dkdv_query_rows: 96, or 80 for head_dim 128 with r_pad 32).
//
// The bias enters the score MMA as R~_k R_q^T with R~_k = R_k*gs/scale, scaled
// in shared memory once per head.  dR_k rides along with dK as extra
// accumulator columns: the B operand of the dK MMA is [Q | R_q] (R_q stored as
// a zero-padded 64-column swizzle atom after Q's), so one N = D + r_pad MMA
// per k-step yields dK and dS^T R_q (dR_k = gs * that).
//
// TMEM columns: dV [0,D) | dK,dR_k [D,2D+r_pad) | S^T (QT) | dP^T (QT) | P^T
// then dS^T (QT/2, packed bf16).  With the packed operands in their own
// columns, the next tile's S^T and dP^T can be computed as soon as the warps
// have read this tile's S^T and dP^T.  P^T and dS^T share their columns: dS^T
// is written once dV has read P^T, the next P^T once dK has read dS^T.
// Per query tile (warpgroup 0 owns query columns [0, QH0), warpgroup 1
// [QH0, QT); each thread one key row = TMEM lane):
//   tensor core:  S^T = K Q^T (+ R~_k R_q^T), dP^T = V dO^T  (SS)
//   warps:        P^T = exp2(S^T*c - LSE2) (bf16), dS^T = P^T (dP^T - Delta)
//   tensor core:  dV += P^T dO, [dK | dR_k] += dS^T [Q | R_q]  (TS form)
// Two threads issue MMAs: one S^T and dP^T, the other dV and dK, so that a
// barrier wait of one stream never sits behind the other stream's queued
// MMAs (a thread's wait issued behind its own queued MMAs only returns once
// the tensor pipe has nearly drained them).
template <int D, int RP>
struct DkdvCfg {
  static constexpr int QT = dkdv_query_rows(D, RP);
  // query columns of warpgroup 0 ([0, QH0)) and 1 ([QH0, QT)): 32 or 48 each, so
  // that every TMEM load and store of a warpgroup starts on a 16-column boundary
  // of its region (80 = 48 + 32)
  static constexpr int QH0 = QT >= 80 ? 48 : 32, QH1 = QT - QH0;
  static constexpr int tDV = 0, tDK = D, tS = 2 * D + RP, tDP = tS + QT, tPT = tDP + QT;
  static_assert(tPT + QT / 2 <= 512, "TMEM budget");
  static_assert((QH0 == 32 || QH0 == 48) && (QH1 == 32 || QH1 == 48), "warpgroup column split");
};

template <int D, int RP>
struct DkdvSmem {
  static constexpr int QT = DkdvCfg<D, RP>::QT;
  static constexpr int kKTile = 128 * D * 2;
  static constexpr int kKChunk = 128 * 128;
  static constexpr int kQChunk = QT * 128;             // one 64-column swizzle atom of a query tile
  static constexpr int kQAtoms = D / 64 + 1;           // Q chunks + the padded R_q atom
  static constexpr int kRk = 128 * RP * 2;
  static constexpr int align(int x) { return (x + 1023) & ~1023; }
  static constexpr int oK = 0;
  static constexpr int oV = align(oK + kKTile);
  static constexpr int oRk = align(oV + kKTile);
  static constexpr int kQStages = 3;                       // Q ring depth (dO: 2)
  static constexpr int kQStage = kQAtoms * kQChunk;         // [Q c0 | (Q c1) | R_q]
  static constexpr int kDoStage = (D / 64) * kQChunk;
  static constexpr int oQ = align(oRk + kRk);
  static constexpr int oDo = oQ + kQStages * kQStage;
  static constexpr int oVec = oDo + 2 * kDoStage;            // per Q stage: [lse2 QT | delta QT] floats
  static constexpr int oBar = oVec + kQStages * 2 * QT * 4;
  static constexpr int kNumBars = 27;
  static constexpr int oMisc = oBar + kNumBars * 8;
  static constexpr int kUsed = oMisc + 16;
  // 1024 bytes of slack for aligning the base when they fit; otherwise the
  // kernel checks that the dynamic shared memory base is 1024-byte aligned
  static constexpr int kTotal = kUsed + 1024 <= kMaxDynamicSmem ? kUsed + 1024 : kUsed;
  static_assert(kUsed <= kMaxDynamicSmem, "shared memory budget");
  static_assert(kQChunk % 1024 == 0, "swizzle atoms need 1024-byte alignment");
};

enum DkdvBar {
  kAKV = 0,
  kARkFull = 1,
  kARkEmpty = 2,
  kAQFull = 3,     // +stage (3): Q and R_q of a query tile
  kAQEmpty = 6,    // +stage (3) (last reader: dK)
  kADoFull = 9,    // +stage (2): dO of a query tile (loaded behind Q)
  kADoEmpty = 11,  // +stage (2) (readers: dP^T and dV, one arrival each)
  kAPrep = 13,     // +stage (3): lse2/Delta rows in shared memory
  kASFull = 16,
  kADPFull = 17,
  kASRead = 18,    // warps have read S^T (one arrival per warp)
  kAPReady = 19,   // P^T in TMEM (one arrival per warp)
  kADsReady = 20,  // dS^T in TMEM (one arrival per warp)
  kADvDone = 21,   // dV MMA of a tile complete (P^T columns free)
  kAHeadDone = 22,
  kAAllDone = 23,
  kARkReady = 24,  // R~_k scaled in shared memory (once per graph head)
  kADpRead = 25,   // warps have read dP^T (one arrival per warp)
  kADkDone = 26,   // dK MMA of a tile complete (dS^T columns free)
};

constexpr int kDkdvThreads = 384;  // 8 softmax-gradient warps, producer, MMA (S/dP), prep, MMA (dV/dK)

// P^T for one chunk of N query columns [qb, qb+N) of one key row:
// exp2(S^T*c - LSE2) into pf[0 .. N); nl holds -LSE2 per query column.  Columns outside [q_lo, q_hi) (causal, sequence end) get exactly 0.
// The fp32 arithmetic runs two columns per packed instruction; each lane is
// rounded as the scalar operation would be.
template <int N>
__device__ __forceinline__ void p_chunk_bwd(const uint32_t* sv_in, float* pf, const int qb, const int q_lo,
                                            const int q_hi, const float* nl, const float sl2) {
  uint32_t sv[N];
#pragma unroll
  for (int k = 0; k < N; ++k) sv[k] = sv_in[k];
  if (!(qb >= q_lo && qb + N <= q_hi)) {
#pragma unroll
    for (int k = 0; k < N; ++k) {  // masked columns: -inf exponent, ex2(-inf) = 0
      const int qi = qb + k;
      if (!(qi >= q_lo && qi < q_hi)) sv[k] = __float_as_uint(-INFINITY);
    }
  }
  const float2 c2 = make_float2(sl2, sl2);
#pragma unroll
  for (int k = 0; k < N; k += 4) {
    const float4 l4 = *reinterpret_cast<const float4*>(&nl[qb + k]);
    const float2 e01 = __ffma2_rn(f32x2(sv[k], sv[k + 1]), c2, make_float2(l4.x, l4.y));
    const float2 e23 = __ffma2_rn(f32x2(sv[k + 2], sv[k + 3]), c2, make_float2(l4.z, l4.w));
    pf[k] = ex2(e01.x), pf[k + 1] = ex2(e01.y), pf[k + 2] = ex2(e23.x), pf[k + 3] = ex2(e23.y);
  }
}

// dS^T = P^T (dP^T - Delta) for N columns starting at query column qb; P^T in
// fp32 (as the reference forms dS), nd holds -Delta per query column, result
// packed into dd.
template <int N>
__device__ __forceinline__ void ds_chunk_bwd(const float* pf, const uint32_t* dp, uint32_t* dd, const int qb,
                                             const float* nd) {
#pragma unroll
  for (int k = 0; k < N; k += 4) {
    const float4 d4 = *reinterpret_cast<const float4*>(&nd[qb + k]);
    const float2 t01 = __fadd2_rn(f32x2(dp[k], dp[k + 1]), make_float2(d4.x, d4.y));
    const float2 t23 = __fadd2_rn(f32x2(dp[k + 2], dp[k + 3]), make_float2(d4.z, d4.w));
    const float2 r01 = __fmul2_rn(make_float2(pf[k], pf[k + 1]), t01);
    const float2 r23 = __fmul2_rn(make_float2(pf[k + 2], pf[k + 3]), t23);
    dd[k >> 1] = pack_bf16(r01.x, r01.y);
    dd[(k >> 1) + 1] = pack_bf16(r23.x, r23.y);
  }
}

// Store a warpgroup's NP packed columns (16, or 24 when it owns 48 query
// columns) of this warp's lanes.
template <int NP>
__device__ __forceinline__ void tmem_st_packed(uint32_t taddr, const uint32_t* r) {
  tmem_st16(taddr, r);
  if constexpr (NP == 24) tmem_st8(taddr + 16, r + 16);
}

// Zero RP accumulator columns of this warp's lanes.
template <int RP>
__device__ __forceinline__ void tmem_zero_cols(uint32_t tcol) {
  uint32_t z[32];
#pragma unroll
  for (int i = 0; i < 32; ++i) z[i] = 0u;
  if (RP == 16) {
    tmem_st16(tcol, z);
  } else {
    tmem_st32(tcol, z);
  }
}

// dR_k of head h from its accumulator columns (cleared at the start of each
// graph head of a GQA group).
template <int RP>
__device__ __forceinline__ void store_drk(const BwdParams& p, const SeqInfo& si, int h, int64_t krow, bool kv_valid,
                                          uint32_t tcol) {
  uint32_t rv[32];
  const ProblemDev& P = p.prob;
  const float gsh = __ldg(P.gs + h);  // dR_k = gs * dS^T R_q
  if (RP == 16) {
    tmem_ld16(tcol, rv);
    tmem_ld_wait16(rv);
  } else {
    tmem_ld32(tcol, rv);
    tmem_ld_wait32(rv);
  }
  if (kv_valid) {
    __nv_bfloat16* dst = p.drk + si.b * p.drk_sb + h * p.drk_sh + krow * p.drk_sr;
#pragma unroll
    for (int c = 0; c < RP; c += 8) {
      if (c < P.rank) {
        uint4 w;
        uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int i = 0; i < 4; ++i)
          wp[i] = pack_bf16(__uint_as_float(rv[c + 2 * i]) * gsh, __uint_as_float(rv[c + 2 * i + 1]) * gsh);
        *reinterpret_cast<uint4*>(dst + c) = w;
      }
    }
  }
}

template <int D, int RP>
__global__ void __launch_bounds__(kDkdvThreads, 1)
    fna2_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDo,
                         const __grid_constant__ CUtensorMap tmRq, const __grid_constant__ CUtensorMap tmRk,
                         const BwdParams p) {
  using L = DkdvSmem<D, RP>;
  using C = DkdvCfg<D, RP>;
  constexpr int QT = C::QT;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  if ((smem - smem_raw) + L::kUsed > L::kTotal) {  // layout does not fit the launch's shared memory
    if (threadIdx.x == 0) atomicCAS(&g_device_error, 0, 499);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::oMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::oMisc + 4);
  float* vec = reinterpret_cast<float*>(smem + L::oVec);

  const ProblemDev& P = p.prob;
  const int hk = grid_head(P);
  int n_blk;
  SeqInfo si;
  if (P.varlen) {  // one CTA per real key tile (table written by the pre kernel)
    const int te = grid_entry(P);
    const int4 e0 = p.tab_k[2 * te], e1 = p.tab_k[2 * te + 1];
    if (e0.x < 0) return;
    n_blk = e0.x;
    si.q_start = e0.y, si.k_start = e0.z, si.len_q = e0.w, si.len_k = e1.x, si.b = 0;
  } else {
    n_blk = blockIdx.x;
    si = seq_info(P, blockIdx.z);
  }
  const int n0 = n_blk * kBlockN;
  if (n0 >= si.len_k) return;
  const int g = P.heads / P.heads_kv;
  const int gh = max(0, min(g, P.heads_graph - hk * g));  // graph heads of this group (a prefix)
  // causal: query tile m sees key rows [n0, n0+128) iff QT*m + QT-1 >= n0
  const int m_start = P.causal ? n0 / QT : 0;
  const int m_end = (si.len_q + QT - 1) / QT;
  const int n_it = max(0, m_end - m_start);
  const int total_it = g * n_it;
  const int warp = warp_id();
  const int lane = lane_id();
  const int tid = threadIdx.x;
  const float scale = P.scale;

  if (total_it == 0) {
    // no query sees this key tile: dK = dV = dR_k = 0
    if (tid < kBlockN && n0 + tid < si.len_k) {
      const int64_t row = si.k_start + n0 + tid;
      zero_row(p.dk + si.b * p.dk_sb + hk * p.dk_sh + row * p.dk_sr, D);
      zero_row(p.dv + si.b * p.dv_sb + hk * p.dv_sh + row * p.dv_sr, D);
      for (int e = 0; e < gh; ++e)
        zero_row(p.drk + si.b * p.drk_sb + (hk * g + e) * p.drk_sh + row * p.drk_sr, P.rank);
    }
    return;
  }

  if (tid == 0) {
    mbar_init(&bars[kAKV], 1);
    mbar_init(&bars[kARkFull], 1);
    mbar_init(&bars[kARkEmpty], 1);
    for (int s = 0; s < L::kQStages; ++s) {
      mbar_init(&bars[kAQFull + s], 1);
      mbar_init(&bars[kAQEmpty + s], 1);
      mbar_init(&bars[kAPrep + s], 32);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kADoFull + s], 1);
      mbar_init(&bars[kADoEmpty + s], 2);  // released by dP^T (stream 1) and dV (stream 2)
    }
    mbar_init(&bars[kASFull], 1);
    mbar_init(&bars[kADPFull], 1);
    mbar_init(&bars[kASRead], 8);
    mbar_init(&bars[kAPReady], 8);
    mbar_init(&bars[kADsReady], 8);
    mbar_init(&bars[kADvDone], 1);
    mbar_init(&bars[kADpRead], 8);
    mbar_init(&bars[kADkDone], 1);
    mbar_init(&bars[kAHeadDone], 1);
    mbar_init(&bars[kAAllDone], 1);
    mbar_init(&bars[kARkReady], 32);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tDV = tmem + C::tDV, tDK = tmem + C::tDK, tS = tmem + C::tS, tDP = tmem + C::tDP,
                 tPT = tmem + C::tPT;
  auto graph_of = [&](int it) { return it / n_it < gh; };

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmDo);
      const int krow = si.k_start + n0;
      mbar_expect_tx(&bars[kAKV], 2 * L::kKTile);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(smem + L::oK + c * L::kKChunk, &tmK, &bars[kAKV], c * 64, krow, hk, si.b);
        tma_load_4d(smem + L::oV + c * L::kKChunk, &tmV, &bars[kAKV], c * 64, krow, hk, si.b);
      }
      int it = 0;
      bool ok = true;
      for (int e = 0; ok && e < g; ++e) {
        const int h = hk * g + e;
        const bool graph = e < gh;
        if (graph) {
          if (e > 0 && !mbar_wait(&bars[kARkEmpty], (e - 1) & 1, abort_flag, 401)) break;
          mbar_expect_tx(&bars[kARkFull], L::kRk);
          tma_load_4d(smem + L::oRk, &tmRk, &bars[kARkFull], 0, krow, h, si.b);
        }
        for (int mi = 0; mi < n_it; ++mi, ++it) {
          const int sq_i = it % L::kQStages, sd = it & 1;
          if (it >= L::kQStages &&
              !mbar_wait(&bars[kAQEmpty + sq_i], ((it / L::kQStages) - 1) & 1, abort_flag, 402)) {
            ok = false;
            break;
          }
          const int qrow = si.q_start + (m_start + mi) * QT;
          uint8_t* sq = smem + L::oQ + sq_i * L::kQStage;
          uint8_t* sdo = smem + L::oDo + sd * L::kDoStage;
          mbar_expect_tx(&bars[kAQFull + sq_i], (D / 64) * L::kQChunk + (graph ? L::kQChunk : 0));
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(sq + c * L::kQChunk, &tmQ, &bars[kAQFull + sq_i], c * 64, qrow, h, si.b);
          if (graph) tma_load_4d(sq + (D / 64) * L::kQChunk, &tmRq, &bars[kAQFull + sq_i], 0, qrow, h, si.b);
          if (it >= 2 && !mbar_wait(&bars[kADoEmpty + sd], ((it >> 1) - 1) & 1, abort_flag, 403)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&bars[kADoFull + sd], (D / 64) * L::kQChunk);
#pragma unroll
          for (int c = 0; c < D / 64; ++c)
            tma_load_4d(sdo + c * L::kQChunk, &tmDo, &bars[kADoFull + sd], c * 64, qrow, h, si.b);
        }
      }
    }
  } else if (warp == 10) {
    // ------------------------------------------------------------ prep: lse2/Delta rows, R~_k
    // the row vectors of tile it+1 are fetched while tile it is staged
    auto fetch = [&](int it, float (&l2)[4], float (&dl)[4]) {
      const int e = it / n_it, mi = it % n_it;
      const int64_t wbase = (static_cast<int64_t>(si.b) * P.heads + hk * g + e) * p.ws_sbh + si.q_start;
      const int m0 = (m_start + mi) * QT;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = lane + 32 * u;
        const bool valid = t < QT && m0 + t < si.len_q;
        l2[u] = valid ? __ldg(p.ws_lse2 + wbase + m0 + t) : 0.f;
        dl[u] = valid ? __ldg(p.ws_delta + wbase + m0 + t) : 0.f;
      }
    };
    float l2[4], dl[4], nl2[4], ndl[4];
    fetch(0, l2, dl);
    bool ok = true;
    for (int it = 0; ok && it < total_it; ++it) {
      const int s = it % L::kQStages;
      const int e = it / n_it;
      if (e < gh && (it % n_it) == 0) {
        // a new graph head: R~_k = R_k * gs/scale in place (element-wise, any swizzle)
        if (!mbar_wait(&bars[kARkFull], e & 1, abort_flag, 652)) {
          ok = false;
          break;
        }
        const float f = __ldg(P.gs + hk * g + e) / scale;
#pragma unroll
        for (int u = 0; u < 4; ++u) scale_rows_inplace<RP>(smem + L::oRk, lane + 32 * u, f);
        fence_proxy_async_smem();
        mbar_arrive(&bars[kARkReady]);
      }
      if (it + 1 < total_it) fetch(it + 1, nl2, ndl);
      // the Q load of tile it implies the stage's previous readers (tile it-3) are done
      if (!mbar_wait(&bars[kAQFull + s], (it / L::kQStages) & 1, abort_flag, 651)) {
        ok = false;
        break;
      }
      float* lv = vec + s * 2 * QT;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (lane + 32 * u < QT) {
          lv[lane + 32 * u] = -l2[u];  // -LSE2 and -Delta: addends of the packed fp32 ops
          lv[QT + lane + 32 * u] = -dl[u];
        }
      }
      mbar_arrive(&bars[kAPrep + s]);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        l2[u] = nl2[u];
        dl[u] = ndl[u];
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA stream 1: S^T, dP^T
    // The whole warp runs the loop and its waits; an elected lane issues each group.
    {
      constexpr uint32_t idesc_st = make_idesc_bf16(128, QT, 0, 0);  // S^T, dP^T (N = QT queries)
      const uint32_t r_layout = r_layout_of(RP);
      const uint32_t r_sbo = 8 * RP * 2;
      const uint32_t sK = smem_u32(smem + L::oK), sV = smem_u32(smem + L::oV), sRk = smem_u32(smem + L::oRk);
      auto stage_q = [&](int it) { return smem_u32(smem + L::oQ + (it % L::kQStages) * L::kQStage); };
      auto issue_s = [&](int it) -> bool {  // S^T = K Q^T (+ R~_k R_q^T)
        const int s = it % L::kQStages;
        const uint32_t par = (it / L::kQStages) & 1;
        if (!mbar_wait_spin(&bars[kAQFull + s], par, abort_flag, 503)) return false;
        if (!mbar_wait_spin(&bars[kAPrep + s], par, abort_flag, 504)) return false;
        if (graph_of(it) && (it % n_it) == 0 &&
            !mbar_wait_spin(&bars[kARkReady], (it / n_it) & 1, abort_flag, 502))
          return false;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t sQ = stage_q(it);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss(tS, make_sdesc(sK + (kk >> 2) * L::kKChunk + (kk & 3) * 32, 16, 1024, kSwizzle128B),
                   make_sdesc(sQ + (kk >> 2) * L::kQChunk + (kk & 3) * 32, 16, 1024, kSwizzle128B), idesc_st, kk > 0);
          if (graph_of(it)) {
            const uint32_t sRq = sQ + (D / 64) * L::kQChunk;
#pragma unroll
            for (int kk = 0; kk < RP / 16; ++kk)
              mma_ss(tS, make_sdesc(sRk + kk * 32, 16, r_sbo, r_layout),
                     make_sdesc(sRq + kk * 32, 16, 1024, kSwizzle128B), idesc_st, 1);
            if ((it % n_it) == n_it - 1) mma_commit(&bars[kARkEmpty]);  // last use of this head's R_k
          }
          mma_commit(&bars[kASFull]);
        }
        __syncwarp();
        return true;
      };
      auto issue_dp = [&](int it) -> bool {  // dP^T = V dO^T
        if (!mbar_wait_spin(&bars[kADoFull + (it & 1)], (it >> 1) & 1, abort_flag, 505)) return false;
        tc_fence_after();
        if (elect_one()) {
          const uint32_t sDo = smem_u32(smem + L::oDo + (it & 1) * L::kDoStage);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            mma_ss(tDP, make_sdesc(sV + (kk >> 2) * L::kKChunk + (kk & 3) * 32, 16, 1024, kSwizzle128B),
                   make_sdesc(sDo + (kk >> 2) * L::kQChunk + (kk & 3) * 32, 16, 1024, kSwizzle128B), idesc_st, kk > 0);
          mma_commit(&bars[kADPFull]);
          mma_commit(&bars[kADoEmpty + (it & 1)]);
        }
        __syncwarp();
        return true;
      };
      bool ok = mbar_wait(&bars[kAKV], 0, abort_flag, 501) && issue_s(0) && issue_dp(0);
      // the next S^T and dP^T as soon as the warps have read this tile's
      for (int it = 0; ok && it + 1 < total_it; ++it)
        ok = mbar_wait_spin(&bars[kASRead], it & 1, abort_flag, 510) && issue_s(it + 1) &&
             mbar_wait_spin(&bars[kADpRead], it & 1, abort_flag, 511) && issue_dp(it + 1);
    }
  } else if (warp == 11) {
    // ------------------------------------------------------------ MMA stream 2: dV, dK
    // The whole warp runs the loop and its waits; an elected lane issues each group.
    {
      constexpr uint32_t idesc_dv = make_idesc_bf16(128, D, 0, 1);        // dV (A in TMEM, B MN-major)
      constexpr uint32_t idesc_dk = make_idesc_bf16(128, D, 0, 1);        // dK only (vanilla heads)
      constexpr uint32_t idesc_dkr = make_idesc_bf16(128, D + RP, 0, 1);  // [dK | dR_k]
      auto stage_q = [&](int it) { return smem_u32(smem + L::oQ + (it % L::kQStages) * L::kQStage); };
      auto stage_do = [&](int it) { return smem_u32(smem + L::oDo + (it & 1) * L::kDoStage); };
      bool ok = true;
      for (int it = 0; ok && it < total_it; ++it) {
        const bool graph = graph_of(it);
        // dV += P^T dO   (K = QT query rows)
        if (!mbar_wait_spin(&bars[kAPReady], it & 1, abort_flag, 506)) break;
        tc_fence_after();
        const uint32_t sDo = stage_do(it), sQ = stage_q(it);
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < QT / 16; ++kk)
            mma_ts(tDV, tPT + 8 * kk, make_sdesc(sDo + kk * 2048, L::kQChunk, 1024, kSwizzle128B), idesc_dv,
                   (it > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&bars[kADvDone]);
          mma_commit(&bars[kADoEmpty + (it & 1)]);
        }
        __syncwarp();
        // [dK | dR_k] += dS^T [Q | R_q]
        if (!mbar_wait_spin(&bars[kADsReady], it & 1, abort_flag, 507)) break;
        tc_fence_after();
        if (elect_one()) {
#pragma unroll
          for (int kk = 0; kk < QT / 16; ++kk)
            mma_ts(tDK, tPT + 8 * kk, make_sdesc(sQ + kk * 2048, L::kQChunk, 1024, kSwizzle128B),
                   graph ? idesc_dkr : idesc_dk, (it > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&bars[kADkDone]);
          mma_commit(&bars[kAQEmpty + it % L::kQStages]);
          if (graph && (it % n_it) == n_it - 1 && it + 1 < total_it) mma_commit(&bars[kAHeadDone]);
        }
        __syncwarp();
      }
      if (ok && elect_one()) mma_commit(&bars[kAAllDone]);
    }
  } else {
    // ------------------------------------------------------------ softmax-gradient warps 0-7
    const int wg = warp >> 2;  // warpgroup: query columns [0, QH0) or [QH0, QT)
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int t = tid & 127;   // key row within the tile (TMEM lane)
    const int kv_local = n0 + t;
    const bool kv_valid = kv_local < si.len_k;
    const float sl2 = P.scale_log2;
    const int64_t krow = si.k_start + kv_local;
    const int qw = wg ? C::QH0 : 0;  // first query column of this warpgroup
    // 48 query columns (else 32); a compile-time constant when both halves match
    const bool wide = wg ? (C::QH1 == 48) : (C::QH0 == 48);
    const uint32_t tSw = tS + lane_base + qw, tDPw = tDP + lane_base + qw;
    const uint32_t tPTw = tPT + lane_base + qw / 2;
    int it = 0, hb = 0;
    bool ok = true;
    // the tile loop, compiled once per column width so that each warpgroup's
    // arrays and loads are sized at compile time
    auto tile_loop = [&](auto wide_tag) {
      constexpr bool kWide = decltype(wide_tag)::value;
      constexpr int QW = kWide ? 48 : 32;  // this warpgroup's query columns
      for (int e = 0; ok && e < g; ++e) {
        const int h = hk * g + e;
        const bool graph = e < gh;
        for (int mi = 0; mi < n_it; ++mi, ++it) {
          const int s = it % L::kQStages;
          const int m0 = (m_start + mi) * QT;
          const float* lv = vec + s * 2 * QT;
          // valid query columns q in [q_lo, q_hi) (tile-relative) for this key row
          const int q_hi = kv_valid ? min(QT, si.len_q - m0) : 0;
          const int q_lo = P.causal ? (kv_local - m0) : 0;
          if (!mbar_wait(&bars[kAPrep + s], (it / L::kQStages) & 1, abort_flag, 702) ||
              !mbar_wait(&bars[kASFull], it & 1, abort_flag, 701)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // phase 1: read S^T, release it for the next tile, then P^T (packed bf16)
          uint32_t sv[QW];
          tmem_ld32(tSw, sv);
          if constexpr (kWide) tmem_ld16(tSw + 32, sv + 32);
          tmem_ld_wait32(sv);
          if constexpr (kWide) tmem_ld_wait16(sv + 32);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[kASRead]);
          float pf[QW];  // P^T in fp32: packed bf16 for the dV MMA, fp32 for dS^T
          p_chunk_bwd<32>(sv, pf, qw, q_lo, q_hi, lv, sl2);
          if constexpr (kWide) p_chunk_bwd<16>(sv + 32, pf + 32, qw + 32, q_lo, q_hi, lv, sl2);
          // the packed columns are free once the previous tile's dK has run
          if (it > 0 && !mbar_wait(&bars[kADkDone], (it - 1) & 1, abort_flag, 703)) {
            ok = false;
            break;
          }
          tc_fence_after();
          {
            uint32_t pk[QW / 2];
#pragma unroll
            for (int k = 0; k < QW / 2; ++k) pk[k] = pack_bf16(pf[2 * k], pf[2 * k + 1]);
            tmem_st_packed<QW / 2>(tPTw, pk);
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[kAPReady]);
          // phase 2: read dP^T (releasing it for the next tile), dS^T = P^T (dP^T - Delta)
          // into the packed columns once dV has read P^T from them
          if (!mbar_wait(&bars[kADPFull], it & 1, abort_flag, 704)) {
            ok = false;
            break;
          }
          tc_fence_after();
          {
            uint32_t dp[QW], dd[QW / 2];
            tmem_ld32(tDPw, dp);
            if constexpr (kWide) tmem_ld16(tDPw + 32, dp + 32);
            tmem_ld_wait32(dp);
            if constexpr (kWide) tmem_ld_wait16(dp + 32);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars[kADpRead]);
            ds_chunk_bwd<QW>(pf, dp, dd, qw, lv + QT);
            if (!mbar_wait(&bars[kADvDone], it & 1, abort_flag, 707)) {
              ok = false;
              break;
            }
            tc_fence_after();
            tmem_st_packed<QW / 2>(tPTw, dd);
          }
          tmem_st_wait();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars[kADsReady]);
          // GQA: at the end of a graph head that is followed by another head, store
          // this head's dR_k columns and clear them for the next head (whose first
          // dK MMA waits for this warpgroup's next dS^T arrival)
          if (wg == 0 && graph && mi == n_it - 1 && it + 1 < total_it) {
            if (!mbar_wait(&bars[kAHeadDone], hb & 1, abort_flag, 705)) {
              ok = false;
              break;
            }
            ++hb;
            tc_fence_after();
            store_drk<RP>(p, si, h, krow, kv_valid, tDK + lane_base + D);
            tmem_zero_cols<RP>(tDK + lane_base + D);
            tmem_st_wait();
            tc_fence_before();
          }
        }
      }
    };
    if (wide)
      tile_loop(std::true_type{});
    else
      tile_loop(std::false_type{});
    if (ok && mbar_wait(&bars[kAAllDone], 0, abort_flag, 706)) {
      tc_fence_after();
      // each warpgroup stores half of the D columns of dV and dK
      // each warpgroup stores half of the D columns of dV and dK, 32 columns at a
      // time, coalesced through the (now idle) Q ring
      constexpr int kCols = D / 2;
      const int row0_local = n0 + (warp & 3) * 32;
      const int64_t row0 = si.k_start + row0_local;
      uint8_t* stage = smem + L::oQ + warp * 32 * 64;
#pragma unroll 1
      for (int mc = 0; mc < 2 * (kCols / 32); ++mc) {  // (dV, dK) x 32-column chunks
        const int m = mc / (kCols / 32), c = mc % (kCols / 32);
        const float f = m == 0 ? 1.f : scale;
        uint32_t v[32], pk[16];
        tmem_ld32((m == 0 ? tDV : tDK) + lane_base + wg * kCols + 32 * c, v);
        tmem_ld_wait32(v);
#pragma unroll
        for (int k = 0; k < 16; ++k)
          pk[k] = pack_bf16(__uint_as_float(v[2 * k]) * f, __uint_as_float(v[2 * k + 1]) * f);
        __nv_bfloat16* dst = m == 0 ? p.dv + si.b * p.dv_sb + hk * p.dv_sh + row0 * p.dv_sr + wg * kCols + 32 * c
                                    : p.dk + si.b * p.dk_sb + hk * p.dk_sh + row0 * p.dk_sr + wg * kCols + 32 * c;
        warp_store_rows<16>(stage, pk, dst, m == 0 ? p.dv_sr : p.dk_sr, si.len_k - row0_local);
      }
      if (wg == 0 && gh > 0 && gh == g) {
        // dR_k of the group's last head (a graph head; otherwise it was stored at its end)
        store_drk<RP>(p, si, hk * g + gh - 1, krow, kv_valid, tDK + lane_base + D);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

constexpr int kQT = dq_key_rows(128, 16);  // key rows per tile of the query-stationary (dQ) kernel

// ---------------------------------------------------------------------------
// dQ / dR_q / d_gs  (Q-stationary)
// ---------------------------------------------------------------------------
// One CTA per (128-row query tile, head, sequence), looping over the causally
// visible 112-row key tiles.  The stationary Q and dO tiles live in tensor
// memory (A operands of the S and dP MMAs in the TS form), which leaves shared
// memory for three-deep K and V rings.  They arrive by TMA in the V ring
// (before its first use) and are moved to tensor memory by tcgen05.cp.
// dR_q rides along with dQ as extra accumulator columns: the B operand of the
// dQ MMA is [K | R_k] (R_k as a zero-padded third 64-column swizzle atom next
// to K's two), so one N = D + r_pad MMA per k-step yields dQ and dS R_k
// together.
// TMEM columns: [dQ | dS R_k] [0,160) S [160,272) dP [272,384) Q [384,448)
// dO [448,512).
// Key tiles are visited from the diagonal down to the first one: the CTAs of
// one head then read different tiles at any moment, so each tile comes from
// HBM once and from L2 for the other CTAs, instead of all of them waiting on
// the same misses in lockstep.
// Per key tile (112 columns; warpgroup 0 owns [0,64), warpgroup 1 [64,112);
// thread = query row = TMEM lane):
//   S = Q K^T (+ R~_q R_k^T) -> warps: P = exp2(S*c - LSE2) in registers
//   dP = dO V^T              -> warps: dS = P (dP - Delta) as bf16 into the
//                               first half of their own dP columns
//   [dQ | dS R_k] += dS [K | R_k]   (TS form)
// The next tile's S is issued as soon as the warps have read S, so it runs
// while they form dS; dQ and the next dP run while they form the next P.
constexpr int kDqStages = 3;

template <int D, int RP>
struct DqSmem {
  static constexpr int kKChunk = kQT * 128;            // one 64-column atom of a 112-row key tile
  static constexpr int kKAtoms = D / 64 + 1;           // K chunks + the padded R_k atom
  static constexpr int kRq = 128 * RP * 2;
  static constexpr int align(int x) { return (x + 1023) & ~1023; }
  static constexpr int oRq = 0;
  static constexpr int oK = align(oRq + kRq);          // stage s: [K c0 | (K c1) | R_k]
  static constexpr int kKStage = kKAtoms * kKChunk;
  static constexpr int oV = oK + kDqStages * kKStage;  // stage s: [V c0 | (V c1)]
  static constexpr int kVStage = (D / 64) * kKChunk;
  static constexpr int kQChunk = 128 * 128;             // one 64-column atom of a 128-row tile
  static constexpr int kQStage = (D / 64) * kQChunk;    // Q (then dO) staged in the V ring
  static_assert(2 * kQStage <= kDqStages * kVStage, "Q and dO must fit in the V ring");
  static constexpr int oBar = align(oV + kDqStages * kVStage);
  static constexpr int kNumBars = 24;
  static constexpr int oMisc = oBar + kNumBars * 8;
  static constexpr int kTotal = oMisc + 16 + 1024;
  static_assert(kKChunk % 1024 == 0, "swizzle atoms need 1024-byte alignment");
};

enum DqBar {
  kBRqFull = 0,   // R_q tile landed (graph heads)
  kBRqReady = 1,  // R~_q scaled (one arrival per warp of warpgroup 0)
  kBKFull = 2,    // +stage
  kBKEmpty = 5,   // +stage
  kBVFull = 8,    // +stage
  kBVEmpty = 11,  // +stage
  kBSFull = 14,
  kBDPFull = 15,
  kBSRead = 16,   // warps have read S (one arrival per warp)
  kBDsReady = 17, // dS in tensor memory (one arrival per warp)
  kBAllDone = 18,
  kBQFull = 19,     // Q and dO tiles landed in the V ring
  kBStageFree = 20, // Q and dO copied to tensor memory; the V ring may be filled
};

constexpr int kDqThreads = 352;  // 8 softmax-gradient warps, producer, MMA issuer, its waiter
constexpr uint32_t kDqHandoffBar = 1;  // named barrier of the issuer / waiter rendezvous

template <int D, int RP>
__global__ void __launch_bounds__(kDqThreads, 1)
    fna2_bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDo,
                       const __grid_constant__ CUtensorMap tmRq, const __grid_constant__ CUtensorMap tmRk,
                       const BwdParams p) {
  using L = DqSmem<D, RP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::oMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::oMisc + 4);

  const ProblemDev& P = p.prob;
  const int h = grid_head(P);
  int m_blk;
  SeqInfo si;
  if (P.varlen) {  // one CTA per real query tile (table written by the pre kernel)
    const int te = grid_entry(P);
    const int4 e0 = p.tab_q[2 * te], e1 = p.tab_q[2 * te + 1];
    if (e0.x < 0) return;
    m_blk = e0.x;
    si.q_start = e0.y, si.k_start = e0.z, si.len_q = e0.w, si.len_k = e1.x, si.b = 0;
  } else {
    m_blk = p.n_mblocks - 1 - static_cast<int>(blockIdx.x);
    si = seq_info(P, blockIdx.z);
  }
  const int q0 = m_blk * kBlockM;
  if (q0 >= si.len_q) return;
  const int hk = h / (P.heads / P.heads_kv);
  const bool graph = h < P.heads_graph;
  const int kv_end = P.causal ? min(si.len_k, q0 + kBlockM) : si.len_k;
  const int n_tiles = kv_end > 0 ? (kv_end + kQT - 1) / kQT : 0;
  const int warp = warp_id();
  const int lane = lane_id();
  const int tid = threadIdx.x;
  const float scale = P.scale;

  if (n_tiles == 0) {
    if (tid < kBlockM && q0 + tid < si.len_q) {
      const int64_t row = si.q_start + q0 + tid;
      zero_row(p.dq + si.b * p.dq_sb + h * p.dq_sh + row * p.dq_sr, D);
      if (graph) zero_row(p.drq + si.b * p.drq_sb + h * p.drq_sh + row * p.drq_sr, P.rank);
    }
    return;
  }

  if (tid == 0) {
    mbar_init(&bars[kBRqFull], 1);
    mbar_init(&bars[kBRqReady], 4);
    mbar_init(&bars[kBQFull], 1);
    mbar_init(&bars[kBStageFree], 1);
    for (int s = 0; s < kDqStages; ++s) {
      mbar_init(&bars[kBKFull + s], 1);
      mbar_init(&bars[kBKEmpty + s], 1);
      mbar_init(&bars[kBVFull + s], 1);
      mbar_init(&bars[kBVEmpty + s], 1);
    }
    mbar_init(&bars[kBSFull], 1);
    mbar_init(&bars[kBDPFull], 1);
    mbar_init(&bars[kBSRead], 8);
    mbar_init(&bars[kBDsReady], 8);
    mbar_init(&bars[kBAllDone], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tDQ = tmem + 0, tS = tmem + 160, tDP = tmem + 272, tQ = tmem + 384, tDO = tmem + 448;
  // TMEM column (relative to dP) of the packed bf16 dS for the 16 keys of k-step kk
  auto packed_col = [](int kk) { return (kk < 4 ? 0 : 64) + (kk & 3) * 8; };

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      const int qrow = si.q_start + q0;
      mbar_expect_tx(&bars[kBQFull], 2 * L::kQStage);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_4d(smem + L::oV + c * L::kQChunk, &tmQ, &bars[kBQFull], c * 64, qrow, h, si.b);
        tma_load_4d(smem + L::oV + L::kQStage + c * L::kQChunk, &tmDo, &bars[kBQFull], c * 64, qrow, h, si.b);
      }
      if (graph) {
        mbar_expect_tx(&bars[kBRqFull], L::kRq);
        tma_load_4d(smem + L::oRq, &tmRq, &bars[kBRqFull], 0, qrow, h, si.b);
      }
      auto load_k = [&](int j) {
        const int s = j % kDqStages;
        const int krow = si.k_start + (n_tiles - 1 - j) * kQT;
        uint8_t* sk = smem + L::oK + s * L::kKStage;
        mbar_expect_tx(&bars[kBKFull + s], (D / 64) * L::kKChunk + (graph ? L::kKChunk : 0));
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sk + c * L::kKChunk, &tmK, &bars[kBKFull + s], c * 64, krow, hk, si.b);
        if (graph) tma_load_4d(sk + (D / 64) * L::kKChunk, &tmRk, &bars[kBKFull + s], 0, krow, h, si.b);
      };
      auto load_v = [&](int j) {
        const int s = j % kDqStages;
        const int krow = si.k_start + (n_tiles - 1 - j) * kQT;
        uint8_t* sv = smem + L::oV + s * L::kVStage;
        mbar_expect_tx(&bars[kBVFull + s], (D / 64) * L::kKChunk);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(sv + c * L::kKChunk, &tmV, &bars[kBVFull + s], c * 64, krow, hk, si.b);
      };
      const int n_first = min(n_tiles, kDqStages);
      for (int j = 0; j < n_first; ++j) load_k(j);
      // the V ring holds the Q and dO tiles until they are in tensor memory
      if (mbar_wait(&bars[kBStageFree], 0, abort_flag, 803)) {
        for (int j = 0; j < n_first; ++j) load_v(j);
        for (int j = kDqStages; j < n_tiles; ++j) {
          const uint32_t par = ((j / kDqStages) - 1) & 1;
          if (!mbar_wait(&bars[kBKEmpty + j % kDqStages], par, abort_flag, 801)) break;
          load_k(j);
          if (!mbar_wait(&bars[kBVEmpty + j % kDqStages], par, abort_flag, 802)) break;
          load_v(j);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp follows the hand-off sequence below; an elected lane
    // issues each group.  It
    // learns that operands are ready only through pair_rendezvous with the
    // waiter warp (warp 10), so it never touches memory behind its queued MMAs.
    constexpr uint32_t idesc_s = make_idesc_bf16(128, kQT, 0, 0);       // S, dP (N = 112 keys)
    constexpr uint32_t idesc_dq = make_idesc_bf16(128, D, 0, 1);        // dQ only (vanilla heads)
    constexpr uint32_t idesc_dqr = make_idesc_bf16(128, D + RP, 0, 1);  // [dQ | dS R_k]
    const uint32_t r_layout = r_layout_of(RP);
    const uint32_t r_sbo = 8 * RP * 2;
    const uint32_t sRq = smem_u32(smem + L::oRq);
    auto stage_k = [&](int j) { return smem_u32(smem + L::oK + (j % kDqStages) * L::kKStage); };
    auto stage_v = [&](int j) { return smem_u32(smem + L::oV + (j % kDqStages) * L::kVStage); };
    auto issue_s = [&](int j) {  // S = Q K^T (+ R~_q R_k^T)
      const uint32_t sK = stage_k(j);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        mma_ts(tS, tQ + kk * 8, make_sdesc(sK + (kk >> 2) * L::kKChunk + (kk & 3) * 32, 16, 1024, kSwizzle128B),
               idesc_s, kk > 0);
      if (graph) {
        const uint32_t sRk = sK + (D / 64) * L::kKChunk;
#pragma unroll
        for (int kk = 0; kk < RP / 16; ++kk)
          mma_ss(tS, make_sdesc(sRq + kk * 32, 16, r_sbo, r_layout), make_sdesc(sRk + kk * 32, 16, 1024, kSwizzle128B),
                 idesc_s, 1);
      }
      mma_commit(&bars[kBSFull]);
    };
    auto issue_dp = [&](int j) {  // dP = dO V^T
      const uint32_t sV = stage_v(j);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk)
        mma_ts(tDP, tDO + kk * 8, make_sdesc(sV + (kk >> 2) * L::kKChunk + (kk & 3) * 32, 16, 1024, kSwizzle128B),
               idesc_s, kk > 0);
      mma_commit(&bars[kBDPFull]);
      mma_commit(&bars[kBVEmpty + (j % kDqStages)]);
    };
    // hand-off 1: Q and dO landed -> shared memory (V ring) to tensor memory, TS A-operand layout
    bool ok = pair_rendezvous(kDqHandoffBar, true);
    if (ok) {
      tc_fence_after();
      if (elect_one()) {
        const uint32_t sQ = smem_u32(smem + L::oV), sDo = sQ + L::kQStage;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kQChunk + (kk & 3) * 32;
          tmem_cp_128x256b(tQ + kk * 8, make_sdesc(sQ + off, 16, 1024, kSwizzle128B));
          tmem_cp_128x256b(tDO + kk * 8, make_sdesc(sDo + off, 16, 1024, kSwizzle128B));
        }
        mma_commit(&bars[kBStageFree]);
      }
      __syncwarp();
    }
    // hand-off 2: R~_q scaled and K(0) landed -> S(0)
    ok = pair_rendezvous(kDqHandoffBar, ok);
    if (ok) {
      tc_fence_after();
      if (elect_one()) issue_s(0);
      __syncwarp();
    }
    // hand-off 3: V(0) landed -> dP(0)
    ok = pair_rendezvous(kDqHandoffBar, ok);
    if (ok) {
      tc_fence_after();
      if (elect_one()) issue_dp(0);
      __syncwarp();
    }
    for (int j = 0; ok && j < n_tiles; ++j) {
      // the warps have read S(j) and K(j+1) landed: next tile's S (it overlaps their dS work)
      ok = pair_rendezvous(kDqHandoffBar, ok);
      if (!ok) break;
      if (j + 1 < n_tiles) {
        tc_fence_after();
        if (elect_one()) issue_s(j + 1);
        __syncwarp();
      }
      // dS(j) written and V(j+1) landed: [dQ | dS R_k] += dS [K | R_k], then the next dP
      ok = pair_rendezvous(kDqHandoffBar, ok);
      if (!ok) break;
      tc_fence_after();
      if (elect_one()) {
        const uint32_t sK = stage_k(j);
#pragma unroll
        for (int kk = 0; kk < kQT / 16; ++kk)
          mma_ts(tDQ, tDP + packed_col(kk), make_sdesc(sK + kk * 2048, L::kKChunk, 1024, kSwizzle128B),
                 graph ? idesc_dqr : idesc_dq, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bars[kBKEmpty + (j % kDqStages)]);
        // next tile's dP (overwrites dS, read in order above)
        if (j + 1 < n_tiles) issue_dp(j + 1);
      }
      __syncwarp();
    }
    if (ok && elect_one()) mma_commit(&bars[kBAllDone]);
  } else if (warp == 10) {
    // ------------------------------------------------------------ waiter for the MMA issuer
    // Same hand-off sequence as warp 9; every wait of the issuer happens here.
    bool ok = mbar_wait(&bars[kBQFull], 0, abort_flag, 901);
    ok = pair_rendezvous(kDqHandoffBar, ok);
    if (ok && graph) ok = mbar_wait(&bars[kBRqReady], 0, abort_flag, 902);
    if (ok) ok = mbar_wait(&bars[kBKFull], 0, abort_flag, 903);
    ok = pair_rendezvous(kDqHandoffBar, ok);
    if (ok) ok = mbar_wait(&bars[kBVFull], 0, abort_flag, 907);
    ok = pair_rendezvous(kDqHandoffBar, ok);
    for (int j = 0; ok && j < n_tiles; ++j) {
      ok = mbar_wait(&bars[kBSRead], j & 1, abort_flag, 904);
      if (ok && j + 1 < n_tiles)
        ok = mbar_wait(&bars[kBKFull + (j + 1) % kDqStages], ((j + 1) / kDqStages) & 1, abort_flag, 905);
      ok = pair_rendezvous(kDqHandoffBar, ok);
      if (!ok) break;
      ok = mbar_wait(&bars[kBDsReady], j & 1, abort_flag, 906);
      if (ok && j + 1 < n_tiles)
        ok = mbar_wait(&bars[kBVFull + (j + 1) % kDqStages], ((j + 1) / kDqStages) & 1, abort_flag, 908);
      ok = pair_rendezvous(kDqHandoffBar, ok);
      if (!ok) break;
    }
  } else {
    // ------------------------------------------------------------ softmax-gradient warps 0-7 (query rows)
    const int wg = warp >> 2;  // key columns [64*wg, min(64*wg+64, 112))
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int t = tid & 127;
    const int q_local = q0 + t;
    const bool row_ok = q_local < si.len_q;
    const int64_t row = si.q_start + q_local;
    const int64_t widx = (static_cast<int64_t>(si.b) * P.heads + h) * p.ws_sbh + row;
    const float lse2 = row_ok ? p.ws_lse2[widx] : 0.f;
    const float delta = row_ok ? p.ws_delta[widx] : 0.f;
    const float sl2 = P.scale_log2;
    // operands of the packed fp32 ops (two columns per instruction)
    const float2 sl2x2 = make_float2(sl2, sl2), nlse2 = make_float2(-lse2, -lse2), ndelta = make_float2(-delta, -delta);
    const int limit = row_ok ? (P.causal ? min(si.len_k, q_local + 1) : si.len_k) : 0;
    bool ok = true;
    // raw R_q row for d_gs, fetched now and used in the epilogue
    uint4 rq_raw[RP / 8];
#pragma unroll
    for (int c = 0; c < RP / 8; ++c) rq_raw[c] = make_uint4(0u, 0u, 0u, 0u);
    if (graph && wg == 0 && row_ok) {
      const uint4* src = reinterpret_cast<const uint4*>(p.rq + si.b * p.rq_sb + h * p.rq_sh + row * p.rq_sr);
#pragma unroll
      for (int c = 0; c < RP / 8; ++c)
        if (8 * c < P.rank) rq_raw[c] = __ldg(src + c);
    }
    if (graph && wg == 0) {
      ok = mbar_wait(&bars[kBRqFull], 0, abort_flag, 1001);
      if (ok) {
        scale_rows_inplace<RP>(smem + L::oRq, t, __ldg(P.gs + h) / scale);
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBRqReady]);
    }
    const uint32_t tSw = tS + lane_base + 64 * wg, tDPw = tDP + lane_base + 64 * wg;
    for (int j = 0; ok && j < n_tiles; ++j) {
      if (!mbar_wait(&bars[kBSFull], j & 1, abort_flag, 1002)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // phase 1 (overlaps the dP MMA): P = exp2(S*c - LSE2) for this warp's keys
      float pf[64];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t sv[32];
        const int col0 = (n_tiles - 1 - j) * kQT + 64 * wg + 32 * c;
        if (c == 0 || wg == 0) {
          tmem_ld32(tSw + 32 * c, sv);
          tmem_ld_wait32(sv);
          if (col0 + 32 > limit) {
#pragma unroll
            for (int k = 0; k < 32; ++k)  // masked key columns: -inf exponent, ex2(-inf) = 0
              if (col0 + k >= limit) sv[k] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float2 e = __ffma2_rn(f32x2(sv[k], sv[k + 1]), sl2x2, nlse2);
            pf[32 * c + k] = ex2(e.x);
            pf[32 * c + k + 1] = ex2(e.y);
          }
        } else {  // warpgroup 1, keys 96..111 of the tile
          tmem_ld16(tSw + 32, sv);
          tmem_ld_wait16(sv);
          if (col0 + 16 > limit) {
#pragma unroll
            for (int k = 0; k < 16; ++k)
              if (col0 + k >= limit) sv[k] = __float_as_uint(-INFINITY);
          }
#pragma unroll
          for (int k = 0; k < 16; k += 2) {
            const float2 e = __ffma2_rn(f32x2(sv[k], sv[k + 1]), sl2x2, nlse2);
            pf[32 + k] = ex2(e.x);
            pf[32 + k + 1] = ex2(e.y);
          }
#pragma unroll
          for (int k = 16; k < 32; ++k) pf[32 + k] = 0.f;
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBSRead]);
      if (!mbar_wait(&bars[kBDPFull], j & 1, abort_flag, 1004)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // phase 2 (overlaps the next S MMA): dS = P (dP - Delta) into this warp's dP columns
      uint32_t dd[32];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t dp[32];
        if (c == 0 || wg == 0) {
          tmem_ld32(tDPw + 32 * c, dp);
          tmem_ld_wait32(dp);
        } else {
          tmem_ld16(tDPw + 32, dp);
          tmem_ld_wait16(dp);
#pragma unroll
          for (int k = 16; k < 32; ++k) dp[k] = 0u;  // beyond the 112-column tile
        }
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const float2 r = __fmul2_rn(make_float2(pf[32 * c + k], pf[32 * c + k + 1]),
                                      __fadd2_rn(f32x2(dp[k], dp[k + 1]), ndelta));
          dd[16 * c + (k >> 1)] = pack_bf16(r.x, r.y);
        }
      }
      tmem_st32(tDPw, dd);  // columns this warp has already read
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBDsReady]);
    }
    if (ok && mbar_wait(&bars[kBAllDone], 0, abort_flag, 1003)) {
      tc_fence_after();
      // each warpgroup stores half of the D columns, through the (now idle) K ring
      constexpr int kCols = D / 2;
      {
        uint32_t pk[kCols / 2];
#pragma unroll
        for (int c = 0; c < kCols / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tDQ + lane_base + wg * kCols + 32 * c, v);
          tmem_ld_wait32(v);
#pragma unroll
          for (int k = 0; k < 16; ++k)
            pk[16 * c + k] = pack_bf16(__uint_as_float(v[2 * k]) * scale, __uint_as_float(v[2 * k + 1]) * scale);
        }
        const int row0_local = q0 + (warp & 3) * 32;
        __nv_bfloat16* dq0 = p.dq + si.b * p.dq_sb + h * p.dq_sh + (si.q_start + row0_local) * p.dq_sr + wg * kCols;
        warp_store_rows<kCols / 2>(smem + L::oK + warp * 32 * kCols * 2, pk, dq0, p.dq_sr, si.len_q - row0_local);
      }
      if (graph && wg == 0) {
        // dR_q = gs * dS R_k (the extra accumulator columns); d_gs += sum_r R_q * dS R_k
        uint32_t rv[32];
        if (RP == 16) {
          tmem_ld16(tDQ + lane_base + D, rv);
          tmem_ld_wait16(rv);
        } else {
          tmem_ld32(tDQ + lane_base + D, rv);
          tmem_ld_wait32(rv);
        }
        float part = 0.f;
        if (row_ok) {
          const float gsh = __ldg(P.gs + h);
          __nv_bfloat16* dst = p.drq + si.b * p.drq_sb + h * p.drq_sh + row * p.drq_sr;
#pragma unroll
          for (int c = 0; c < RP; c += 8) {
            if (c >= P.rank) break;
            const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rq_raw[c / 8]);
            uint4 w;
            uint32_t* wp = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const float a0 = __uint_as_float(rv[c + 2 * i]), a1 = __uint_as_float(rv[c + 2 * i + 1]);
              const float2 rr = __bfloat1622float2(r2[i]);
              part = fmaf(rr.x, a0, part);
              part = fmaf(rr.y, a1, part);
              wp[i] = pack_bf16(a0 * gsh, a1 * gsh);
            }
            *reinterpret_cast<uint4*>(dst + c) = w;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (lane == 0) atomicAdd(p.dgs + h, part);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// host-side launch (called from fna2_api.cu)
// ---------------------------------------------------------------------------
template <int D, int RP>
cudaError_t launch_bwd_t(const BwdMaps& m, const BwdParams& p, cudaStream_t stream, cudaEvent_t* ev) {
  const int bdim = p.prob.varlen ? 1 : p.batch;
  if (ev) {
    cudaError_t e = cudaEventRecord(ev[0], stream);
    if (e != cudaSuccess) return e;
  }
  {
    const int rows = max(p.total_q_rows, p.total_k_rows);
    dim3 grid((rows + 127) / 128, p.prob.heads, bdim);
    fna2_bwd_pre_kernel<D><<<grid, 128, 0, stream>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess && ev) e = cudaEventRecord(ev[1], stream);
    if (e != cudaSuccess) return e;
  }
  {
    using L = DkdvSmem<D, RP>;
    auto kern = fna2_bwd_dkdv_kernel<D, RP>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (e != cudaSuccess) return e;
    dim3 grid(p.prob.varlen ? p.tab_k_len : p.n_nblocks, p.prob.heads_kv, p.prob.varlen ? 1 : p.batch);
    if (p.prob.varlen && p.prob.head_fast) grid = dim3(p.prob.heads_kv, p.tab_k_len, 1);
    kern<<<grid, kDkdvThreads, L::kTotal, stream>>>(m.qS, m.k, m.v, m.dOS, m.rqS, m.rk, p);
    e = cudaGetLastError();
    if (e == cudaSuccess && ev) e = cudaEventRecord(ev[2], stream);
    if (e != cudaSuccess) return e;
  }
  {
    using L = DqSmem<D, RP>;
    auto kern = fna2_bwd_dq_kernel<D, RP>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
    if (e != cudaSuccess) return e;
    dim3 grid(p.prob.varlen ? p.tab_q_len : p.n_mblocks, p.prob.heads, p.prob.varlen ? 1 : p.batch);
    if (p.prob.varlen && p.prob.head_fast) grid = dim3(p.prob.heads, p.tab_q_len, 1);
    kern<<<grid, kDqThreads, L::kTotal, stream>>>(m.q, m.kDq, m.vDq, m.dO, m.rq, m.rkDq, p);
    e = cudaGetLastError();
    if (e == cudaSuccess && ev) e = cudaEventRecord(ev[3], stream);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t launch_bwd(int D, int RP, const BwdMaps& m, const BwdParams& p, cudaStream_t stream, cudaEvent_t* ev) {
  if (D == 64 && RP == 16) return launch_bwd_t<64, 16>(m, p, stream, ev);
  if (D == 64 && RP == 32) return launch_bwd_t<64, 32>(m, p, stream, ev);
  if (D == 128 && RP == 16) return launch_bwd_t<128, 16>(m, p, stream, ev);
  if (D == 128 && RP == 32) return launch_bwd_t<128, 32>(m, p, stream, ev);
  return cudaErrorInvalidValue;
}

}  // namespace fna2

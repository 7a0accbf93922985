// FNA2 forward on sm_100a: O = softmax(scale*Q K^T + gs*R_q R_k^T [causal]) V
// and LSE, dense [B,H,S,D] and varlen [T,H,D] through the same kernel.
//
// Reference semantics: FNA2/flash_naylis_attn.py:58-201 (dense) and :208-349
// (varlen): bias only on graph heads h < H_G, GQA kv_head = h / (H/H_KV),
// causal on sequence-local positions, O = acc/(l+1e-6), LSE = m + log(l+1e-6).
//
// Design: one CTA per pair of 128-row query tiles (256 rows) of one head and
// sequence, so that every K/V tile brought into shared memory feeds two score
// tiles and two softmax warpgroups share each SM sub-partition's exp2 units.
//   warps 0-3 / 4-7  softmax of query tile 0 / 1: thread t owns query row t
//              of its tile = TMEM lane t.  Reads the 128x128 fp32 score tile
//              from TMEM, applies masks, keeps the running max/sum in
//              registers, writes P (bf16) back into the same TMEM columns,
//              rescales O in TMEM only when the max grew by more than 2^8
//              (exactly compensated at the end).
//   warp 8     TMA producer: Q and R_q of both tiles once; K(+R_k) and V
//              tiles through two separate 2-stage mbarrier rings.
//   warp 9     allocates 512 TMEM columns; one thread issues tcgen05.mma:
//                S_i  = Q_i K^T + R~_q,i R_k^T (SS, K = D + r_pad; the bias is
//                       an extra K slice, R~_q = R_q * gs/scale in smem)
//                O_i += P_i V                  (TS, P read from TMEM)
//              in the order O_0 += P_0 V(j), S_0(j+1), O_1 += P_1 V(j),
//              S_1(j+1): while one warpgroup turns S into P the tensor core
//              works on the other tile.
// TMEM columns: O_0 [0,128), O_1 [128,256), S_0 [256,384), S_1 [384,512).
// S_i(j+1) overwrites P_i(j) only after O_i += P_i(j) V(j) (same issuing
// thread, in order), and the commit that signals S_i(j+1) also covers
// O_i += P_i(j) V(j), so a warpgroup that sees S_i(j+1) may rescale O_i.
#include "fna2_kernels.cuh"
#include "ptx.cuh"

namespace fna2 {

constexpr int kFwdTiles = 2;  // 128-row query tiles per CTA

template <int D, int RP>
struct FwdSmem {
  static constexpr int kQBytes = kBlockM * D * 2;
  static constexpr int kRqBytes = kBlockM * RP * 2;
  static constexpr int kKBytes = kBlockN * D * 2;
  static constexpr int kRkBytes = kBlockN * RP * 2;
  static constexpr int kVBytes = kBlockN * D * 2;
  static constexpr int kChunk = 128 * 128;  // one 64-column chunk of a 128-row tile (bytes)
  static constexpr int align(int x) { return (x + 1023) & ~1023; }
  static constexpr int oQ = 0;                                    // Q_0, Q_1
  static constexpr int oRq = align(oQ + kFwdTiles * kQBytes);     // R~_q,0, R~_q,1
  static constexpr int oK0 = align(oRq + kFwdTiles * kRqBytes);
  static constexpr int oK1 = align(oK0 + kKBytes);
  static constexpr int oRk0 = align(oK1 + kKBytes);
  static constexpr int oRk1 = align(oRk0 + kRkBytes);
  static constexpr int oV0 = align(oRk1 + kRkBytes);
  static constexpr int oV1 = align(oV0 + kVBytes);
  static constexpr int oBar = align(oV1 + kVBytes);
  static constexpr int kNumBars = 20;
  static constexpr int oMisc = oBar + kNumBars * 8;
  static constexpr int kUsed = oMisc + 16;
  // 1024 bytes of slack for aligning the base when they fit; otherwise the
  // kernel checks that the dynamic shared memory base is 1024-byte aligned
  static constexpr int kTotal = kUsed + 1024 <= kMaxDynamicSmem ? kUsed + 1024 : kUsed;
  static_assert(kUsed <= kMaxDynamicSmem, "shared memory budget");
};

enum FwdBar {
  kBarQFull = 0,
  kBarRqReady = 1,   // +tile: R~_q,i scaled (one arrival per warp of warpgroup i)
  kBarKFull = 3,     // +stage
  kBarKEmpty = 5,    // +stage
  kBarVFull = 7,     // +stage
  kBarVEmpty = 9,    // +stage
  kBarSFull = 11,    // +tile
  kBarPFull = 13,    // +tile (one arrival per warp)
  kBarAllDone = 15,
};

constexpr int kFwdThreads = 320;  // 2 softmax warpgroups, producer, MMA

// Epilogue: this warp's 32 rows of O (TMEM, fp32) times inv, as bf16, 32
// columns at a time through a 2 KB shared-memory staging buffer.  Kept out of
// line so that the softmax loop's register allocation does not see it.
template <int D>
__device__ __noinline__ void store_o_rows(uint8_t* stage, uint32_t tO, float inv, __nv_bfloat16* o0,
                                          int64_t row_stride, int nvalid) {
#pragma unroll 1
  for (int c = 0; c < D / 32; ++c) {
    uint32_t o[32], pk[16];
    tmem_ld32(tO + 32 * c, o);
    tmem_ld_wait32(o);
#pragma unroll
    for (int k = 0; k < 16; ++k) pk[k] = pack_bf16(__uint_as_float(o[2 * k]) * inv, __uint_as_float(o[2 * k + 1]) * inv);
    warp_store_rows<16>(stage, pk, o0 + 32 * c, row_stride, nvalid);
  }
}

template <int D, int RP>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fna2_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmRq,
                    const __grid_constant__ CUtensorMap tmRk, const FwdParams p) {
  using L = FwdSmem<D, RP>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  if ((smem - smem_raw) + L::kUsed > L::kTotal) {  // layout does not fit the launch's shared memory
    if (threadIdx.x == 0) atomicCAS(&g_device_error, 0, 199);
    return;
  }
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::oMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::oMisc + 4);

  const ProblemDev& P = p.prob;
  int pair;
  SeqInfo si;
  if (P.varlen) {
    // grid (table entry, head): one CTA per real pair of query tiles; the table
    // lists each sequence's pairs heaviest first, so the CTAs of one head and
    // sequence run together and share its K/V tiles in L2 (head_fast: the
    // transposed grid of small problems)
    const int te = grid_entry(P);
    const int4 e0 = p.tab[2 * te], e1 = p.tab[2 * te + 1];
    if (e0.x < 0) return;
    pair = e0.x;
    si.q_start = e0.y, si.k_start = e0.z, si.len_q = e0.w, si.len_k = e1.x, si.b = 0;
  } else {  // grid (pair, head, batch), heaviest causal pairs first
    pair = (p.n_mblocks + 1) / 2 - 1 - static_cast<int>(blockIdx.x);
    si = seq_info(P, blockIdx.z);
  }
  const int h = grid_head(P);
  const int q0 = pair * 2 * kBlockM;
  if (q0 >= si.len_q) return;
  const int hk = h / (P.heads / P.heads_kv);
  const bool graph = h < P.heads_graph;
  // key tiles seen by each query tile (0 when the tile has no query row)
  int n_t[kFwdTiles];
#pragma unroll
  for (int i = 0; i < kFwdTiles; ++i) {
    const int qt = q0 + i * kBlockM;
    const int kv_end = qt >= si.len_q ? 0 : (P.causal ? min(si.len_k, qt + kBlockM) : si.len_k);
    n_t[i] = kv_end > 0 ? (kv_end + kBlockN - 1) / kBlockN : 0;
  }
  const int n_kv = max(n_t[0], n_t[1]);
  const int warp = warp_id();
  const int lane = lane_id();
  const int tid = threadIdx.x;

  if (n_kv == 0) {
    // No visible key: the reference's loop is empty, O = 0 and LSE = -inf.
    if (tid < kFwdTiles * kBlockM && q0 + tid < si.len_q) {
      const int row = si.q_start + q0 + tid;
      __nv_bfloat16* orow = p.out + si.b * p.o_sb + h * p.o_sh + static_cast<int64_t>(row) * p.o_sr;
      for (int c = 0; c < D; ++c) orow[c] = __float2bfloat16(0.f);
      p.lse[(static_cast<int64_t>(si.b) * P.heads + h) * p.lse_sbh + row] = -INFINITY;
    }
    return;
  }

  if (tid == 0) {
    mbar_init(&bars[kBarQFull], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[kBarRqReady + s], 4);
      mbar_init(&bars[kBarKFull + s], 1);
      mbar_init(&bars[kBarKEmpty + s], 1);
      mbar_init(&bars[kBarVFull + s], 1);
      mbar_init(&bars[kBarVEmpty + s], 1);
      mbar_init(&bars[kBarSFull + s], 1);
      mbar_init(&bars[kBarPFull + s], 4);
    }
    mbar_init(&bars[kBarAllDone], 1);
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

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      if (graph) {
        tma_prefetch_desc(&tmRq);
        tma_prefetch_desc(&tmRk);
      }
      int q_bytes = 0;
#pragma unroll
      for (int i = 0; i < kFwdTiles; ++i)
        if (n_t[i] > 0) q_bytes += L::kQBytes + (graph ? L::kRqBytes : 0);
      mbar_expect_tx(&bars[kBarQFull], q_bytes);
#pragma unroll
      for (int i = 0; i < kFwdTiles; ++i) {
        if (n_t[i] == 0) continue;
        const int qrow = si.q_start + q0 + i * kBlockM;
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(smem + L::oQ + i * L::kQBytes + c * L::kChunk, &tmQ, &bars[kBarQFull], c * 64, qrow, h, si.b);
        if (graph) tma_load_4d(smem + L::oRq + i * L::kRqBytes, &tmRq, &bars[kBarQFull], 0, qrow, h, si.b);
      }

      auto load_k = [&](int j) -> bool {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bars[kBarKEmpty + s], ((j >> 1) - 1) & 1, abort_flag, 101)) return false;
        uint8_t* dk = smem + (s ? L::oK1 : L::oK0);
        const int krow = si.k_start + j * kBlockN;
        mbar_expect_tx(&bars[kBarKFull + s], L::kKBytes + (graph ? L::kRkBytes : 0));
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(dk + c * L::kChunk, &tmK, &bars[kBarKFull + s], c * 64, krow, hk, si.b);
        if (graph) tma_load_4d(smem + (s ? L::oRk1 : L::oRk0), &tmRk, &bars[kBarKFull + s], 0, krow, h, si.b);
        return true;
      };
      auto load_v = [&](int j) -> bool {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&bars[kBarVEmpty + s], ((j >> 1) - 1) & 1, abort_flag, 102)) return false;
        uint8_t* dv = smem + (s ? L::oV1 : L::oV0);
        const int krow = si.k_start + j * kBlockN;
        mbar_expect_tx(&bars[kBarVFull + s], L::kVBytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_4d(dv + c * L::kChunk, &tmV, &bars[kBarVFull + s], c * 64, krow, hk, si.b);
        return true;
      };
      bool ok = load_k(0);
      if (ok && n_kv > 1) ok = load_k(1);
      for (int j = 0; ok && j < n_kv; ++j) {
        ok = load_v(j);
        if (ok && j + 2 < n_kv) ok = load_k(j + 2);
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------------ MMA issuer
    // The whole warp runs the loop and its waits; an elected lane issues each group.
    {
      constexpr uint32_t idesc_s = make_idesc_bf16(kBlockM, kBlockN, 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_bf16(kBlockM, D, 0, 1);
      constexpr uint32_t r_layout = RP == 16 ? kSwizzle32B : (RP == 32 ? kSwizzle64B : kSwizzle128B);
      constexpr uint32_t r_sbo = 8 * RP * 2;
      bool ok = mbar_wait(&bars[kBarQFull], 0, abort_flag, 201);
#pragma unroll
      for (int i = 0; i < kFwdTiles; ++i)
        if (ok && graph && n_t[i] > 0) ok = mbar_wait(&bars[kBarRqReady + i], 0, abort_flag, 202);

      // S_i(j) = Q_i K(j)^T (+ R~_q,i R_k(j)^T); the last user of K(j) releases its stage
      auto issue_s = [&](int i, int j) {
        const int b = j & 1;
        const uint32_t sQ = smem_u32(smem + L::oQ + i * L::kQBytes);
        const uint32_t sK = smem_u32(smem + (b ? L::oK1 : L::oK0));
        const uint32_t tS = tmem + 256 + 128 * i;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kChunk + (kk & 3) * 32;
          mma_ss(tS, make_sdesc(sQ + off, 16, 1024, kSwizzle128B), make_sdesc(sK + off, 16, 1024, kSwizzle128B),
                 idesc_s, kk > 0);
        }
        if (graph) {
          const uint32_t sRq = smem_u32(smem + L::oRq + i * L::kRqBytes);
          const uint32_t sRk = smem_u32(smem + (b ? L::oRk1 : L::oRk0));
#pragma unroll
          for (int kk = 0; kk < RP / 16; ++kk)
            mma_ss(tS, make_sdesc(sRq + kk * 32, 16, r_sbo, r_layout), make_sdesc(sRk + kk * 32, 16, r_sbo, r_layout),
                   idesc_s, 1);
        }
        mma_commit(&bars[kBarSFull + i]);
        if (i == 1 || j >= n_t[1]) mma_commit(&bars[kBarKEmpty + b]);
      };
      auto wait_k = [&](int j) -> bool {
        if (!mbar_wait_spin(&bars[kBarKFull + (j & 1)], (j >> 1) & 1, abort_flag, 203)) return false;
        tc_fence_after();
        return true;
      };

      if (ok) ok = wait_k(0);
      if (ok) {
        if (elect_one()) {
#pragma unroll
          for (int i = 0; i < kFwdTiles; ++i)
            if (n_t[i] > 0) issue_s(i, 0);
        }
        __syncwarp();
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int b = j & 1;
        const uint32_t sV = smem_u32(smem + (b ? L::oV1 : L::oV0));
        if (!mbar_wait_spin(&bars[kBarVFull + b], (j >> 1) & 1, abort_flag, 205)) break;
        if (j + 1 < n_kv && !wait_k(j + 1)) break;
#pragma unroll
        for (int i = 0; i < kFwdTiles; ++i) {
          if (j >= n_t[i]) continue;
          // O_i += P_i(j) V(j), then S_i(j+1) over the same TMEM columns
          if (!mbar_wait_spin(&bars[kBarPFull + i], (j & 1), abort_flag, 204)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (elect_one()) {
            const uint32_t tO = tmem + 128 * i;
            const uint32_t tP = tmem + 256 + 128 * i;
#pragma unroll
            for (int kk = 0; kk < kBlockN / 16; ++kk)
              mma_ts(tO, tP + kk * 8, make_sdesc(sV + kk * 2048, L::kChunk, 1024, kSwizzle128B), idesc_pv,
                     (j > 0 || kk > 0) ? 1u : 0u);
            if (j + 1 < n_t[i]) issue_s(i, j + 1);
          }
          __syncwarp();
        }
        if (elect_one()) mma_commit(&bars[kBarVEmpty + b]);
        __syncwarp();
      }
      if (ok && elect_one()) mma_commit(&bars[kBarAllDone]);
    }
  } else {
    // ------------------------------------------------------------ softmax (warpgroup i = query tile i)
    const int wi = warp >> 2;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tO = tmem + 128 * wi + lane_base;
    const uint32_t tSrow = tmem + 256 + 128 * wi + lane_base;
    const int t = tid & 127;
    const int q_local = q0 + wi * kBlockM + t;
    const int n_my = wi ? n_t[1] : n_t[0];
    const float sl2 = P.scale_log2;
    bool ok = true;
    // watchdog test hook: tile 0 withholds its first P hand-off (never set in normal use)
    const bool withhold = wi == 0 && *reinterpret_cast<volatile int*>(&g_debug_withhold) == kSiteFwdPFull;

    if (graph && n_my > 0) {
      // R~_q = R_q * gs/scale in place (element-wise, so independent of the swizzle).
      ok = mbar_wait(&bars[kBarQFull], 0, abort_flag, 301);
      if (ok) {
        const float f = __ldg(P.gs + h) / P.scale;
        uint4* rrow = reinterpret_cast<uint4*>(smem + L::oRq + wi * L::kRqBytes + t * RP * 2);
#pragma unroll
        for (int u = 0; u < RP / 8; ++u) {
          uint4 w = rrow[u];
          uint32_t* e = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            __nv_bfloat162 v2 = *reinterpret_cast<__nv_bfloat162*>(&e[k]);
            float2 f2 = __bfloat1622float2(v2);
            e[k] = pack_bf16(f2.x * f, f2.y * f);
          }
          rrow[u] = w;
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[kBarRqReady + wi]);
    }

    const int limit = P.causal ? min(si.len_k, q_local + 1) : si.len_k;
    float m_use = -INFINITY, m_true = -INFINITY, l = 0.f;
    uint32_t r[128];
    for (int j = 0; ok && j < n_my; ++j) {
      if (!mbar_wait(&bars[kBarSFull + wi], j & 1, abort_flag, 302)) {
        ok = false;
        break;
      }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tSrow + 32 * c, r + 32 * c);
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_wait32(r + 32 * c);

      const int nvalid = limit - j * kBlockN;
      // row max with 8 independent chains (a single chain of 128 dependent
      // fmaxf would dominate the tile's latency)
      float m8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) m8[k] = -INFINITY;
      if (nvalid >= kBlockN) {
#pragma unroll
        for (int k = 0; k < 128; ++k) m8[k & 7] = fmaxf(m8[k & 7], __uint_as_float(r[k]));
      } else {
#pragma unroll
        for (int k = 0; k < 128; ++k) {
          const float x = k < nvalid ? __uint_as_float(r[k]) : -INFINITY;
          r[k] = __float_as_uint(x);
          m8[k & 7] = fmaxf(m8[k & 7], x);
        }
      }
      float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
      mx *= sl2;
      m_true = fmaxf(m_true, mx);
      float alpha = 1.f;
      bool rescale = false;
      if (m_true - m_use > 8.f || m_use == -INFINITY) {
        // grow the reference max; O (if any) must be scaled by alpha
        alpha = (m_use == -INFINITY) ? 0.f : ex2(m_use - m_true);
        rescale = (j > 0);
        m_use = m_true;
      }
      const float mb = (m_use == -INFINITY) ? 0.f : m_use;
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};  // independent partial sums
#pragma unroll
      for (int k = 0; k < 128; k += 2) {
        const float p0 = ex2(fmaf(__uint_as_float(r[k]), sl2, -mb));
        const float p1 = ex2(fmaf(__uint_as_float(r[k + 1]), sl2, -mb));
        rs4[(k >> 1) & 3] += p0 + p1;
        r[k >> 1] = pack_bf16(p0, p1);
      }
      l = l * alpha + ((rs4[0] + rs4[1]) + (rs4[2] + rs4[3]));
      // P (bf16 pairs) over the first 64 columns of this S buffer
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_st16(tSrow + 16 * c, r + 16 * c);
      // O_i += P_i(j-1) V(j-1) is complete (covered by the S_i(j) commit): rescale O_i if needed
      if (j > 0 && __any_sync(0xffffffffu, rescale)) {
        const float a = rescale ? alpha : 1.f;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + 32 * c, o);
          tmem_ld_wait32(o);
#pragma unroll
          for (int k = 0; k < 32; ++k) o[k] = __float_as_uint(__uint_as_float(o[k]) * a);
          tmem_st32(tO + 32 * c, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0 && !(withhold && j == 0)) mbar_arrive(&bars[kBarPFull + wi]);
    }

    if (ok && n_my > 0 && mbar_wait(&bars[kBarAllDone], 0, abort_flag, 304)) {
      tc_fence_after();
      // exact reference normalisation with the true running max
      const float corr = (m_use == -INFINITY) ? 0.f : ex2(m_use - m_true);
      const float l_true = l * corr;
      const float inv = corr / (l_true + kEps);
      const bool row_ok = q_local < si.len_q;
      const int row = si.q_start + q_local;
      // O rows, 32 columns at a time, coalesced through the (now idle) K ring
      const int row0_local = q0 + wi * kBlockM + (warp & 3) * 32;
      __nv_bfloat16* o0 = p.out + si.b * p.o_sb + h * p.o_sh + static_cast<int64_t>(si.q_start + row0_local) * p.o_sr;
      store_o_rows<D>(smem + L::oK0 + warp * 32 * 64, tO, inv, o0, p.o_sr, si.len_q - row0_local);
      if (row_ok) {
        const float lse = (m_true == -INFINITY) ? -INFINITY : (m_true + lg2(l_true + kEps)) * kLn2;
        p.lse[(static_cast<int64_t>(si.b) * P.heads + h) * p.lse_sbh + row] = lse;
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
// varlen: table of the real pairs of query tiles (one CTA, before the forward)
// ---------------------------------------------------------------------------
// Entries per sequence, in packing order, heaviest causal pair first.  A
// sequence whose cu_seqlens entries are inconsistent (seq_ok) gets no entries
// and the call records kStatusBadSeqFwd.  A block-wide scan runs over chunks of
// 128 sequences, carrying the running offset from chunk to chunk.
inline int fwd_tab_len(int rows_q, int n_seqs) { return (rows_q + 2 * kBlockM - 1) / (2 * kBlockM) + n_seqs; }

inline size_t fwd_workspace_bytes(bool varlen, int rows_q, int n_seqs) {
  return varlen ? static_cast<size_t>(fwd_tab_len(rows_q, n_seqs)) * 32 : 0;
}

__global__ void __launch_bounds__(128) fna2_fwd_table_kernel(const FwdParams p, int n_seqs) {
  const ProblemDev& P = p.prob;
  __shared__ int scan_s[4];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int carry = 0;
  for (int base = 0; base < n_seqs; base += 128) {
    const int z = base + static_cast<int>(threadIdx.x);
    SeqInfo e;
    e.q_start = e.k_start = e.len_q = e.len_k = 0;
    e.b = 0;
    if (z < n_seqs) {
      e.q_start = __ldg(P.cu_q + z), e.len_q = __ldg(P.cu_q + z + 1) - e.q_start;
      e.k_start = __ldg(P.cu_k + z), e.len_k = __ldg(P.cu_k + z + 1) - e.k_start;
      if (!seq_ok(P, e)) {  // skipped before any access; reported once per call
        atomicCAS(&g_device_error, 0, kStatusBadSeqFwd);
        e.len_q = 0;
      }
    }
    const int np = (e.len_q + 2 * kBlockM - 1) / (2 * kBlockM);  // >= 0
    int incl = np;  // inclusive scan within the warp
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) scan_s[w] = incl;
    __syncthreads();
    int off = carry + incl - np;
    for (int i = 0; i < w; ++i) off += scan_s[i];
    for (int t = 0; t < np && off + t < p.tab_len; ++t) {
      p.tab[2 * (off + t)] = make_int4(np - 1 - t, e.q_start, e.k_start, e.len_q);
      p.tab[2 * (off + t) + 1] = make_int4(e.len_k, z, 0, 0);
    }
    carry += scan_s[0] + scan_s[1] + scan_s[2] + scan_s[3];
    __syncthreads();
  }
  for (int i = carry + static_cast<int>(threadIdx.x); i < p.tab_len; i += 128) p.tab[2 * i] = make_int4(-1, 0, 0, 0);
}

// ---------------------------------------------------------------------------
// host-side launch helper (called from fna2_api.cu)
// ---------------------------------------------------------------------------
template <int D, int RP>
cudaError_t launch_fwd_t(const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v, const CUtensorMap& rq,
                         const CUtensorMap& rk, const FwdParams& p, int grid_y, int grid_z, cudaStream_t stream) {
  using L = FwdSmem<D, RP>;
  auto kern = fna2_fwd_kernel<D, RP>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kTotal);
  if (e != cudaSuccess) return e;
  if (p.prob.varlen) {
    fna2_fwd_table_kernel<<<1, 128, 0, stream>>>(p, grid_z);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  const dim3 grid = !p.prob.varlen         ? dim3((p.n_mblocks + 1) / 2, grid_y, grid_z)
                    : p.prob.head_fast ? dim3(grid_y, p.tab_len, 1)
                                       : dim3(p.tab_len, grid_y, 1);
  kern<<<grid, kFwdThreads, L::kTotal, stream>>>(q, k, v, rq, rk, p);
  return cudaGetLastError();
}

cudaError_t launch_fwd(int D, int RP, const CUtensorMap& q, const CUtensorMap& k, const CUtensorMap& v,
                       const CUtensorMap& rq, const CUtensorMap& rk, const FwdParams& p, int grid_y, int grid_z,
                       cudaStream_t stream) {
  if (D == 64 && RP == 16) return launch_fwd_t<64, 16>(q, k, v, rq, rk, p, grid_y, grid_z, stream);
  if (D == 64 && RP == 32) return launch_fwd_t<64, 32>(q, k, v, rq, rk, p, grid_y, grid_z, stream);
  if (D == 128 && RP == 16) return launch_fwd_t<128, 16>(q, k, v, rq, rk, p, grid_y, grid_z, stream);
  if (D == 128 && RP == 32) return launch_fwd_t<128, 32>(q, k, v, rq, rk, p, grid_y, grid_z, stream);
  return cudaErrorInvalidValue;
}

}  // namespace fna2

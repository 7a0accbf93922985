// Dense bf16 GEMM on tcgen05 for the stacked R_q/R_k projection (row f2):
//   C[m][n] = sum_k A[m][k] * B[n][k]        (fp32 accumulation in TMEM)
// with each operand stored either K-major (A[m][k] at a[m*lda + k]) or
// MN-major (A[m][k] at a[k*lda + m]), so one kernel serves the projection's
// three products (FNA2/attention_fna2.py:320-335 is the forward the reference
// runs as two nn.Linear layers; autograd adds the two others):
//   forward  Y  = X W^T      A = X  (K-major)   B = W  (K-major)   C bf16
//   dX       dX = dY W       A = dY (K-major)   B = W  (MN-major)  C bf16
//   dW       dW = dY^T X     A = dY (MN-major)  B = X  (MN-major)  C fp32, split over K
// The dW product reduces over all T tokens: with fp32 output the K range may
// be split into slices (work items ordered slice-major, so that the CTAs
// running together read the same K chunks and share them in L2), and the
// partial tiles are added into C (the caller clears it) with red.global.add.
//
// A cluster of two CTAs computes a 256 x 256 output tile with M = 256 MMAs over
// the pair (tcgen05 cta_group::2): CTA r loads A's rows [128r, 128r+128) and B's
// rows (output columns) [128r, 128r+128) of the tile, and each MMA reads both
// CTAs' halves, so each CTA loads 32 KB per 64-deep K chunk for the work that a
// single-CTA 128 x 256 tile needs 48 KB for (shared-memory traffic, not the
// tensor pipe, bounds the single-CTA form).  Persistent: each pair takes work
// items (output tile, K slice) round-robin, output tiles N-fastest so that the
// pairs running together share A's rows in L2.  Per CTA: warp 0 loads chunks
// by TMA into a 6-stage ring that runs on across items, completion counted on
// the even CTA's barriers (the even CTA registers both CTAs' bytes with one
// local arrival: a cluster-scope arrival from the odd CTA per chunk made its
// producer the bottleneck, 20.0 against 10.9 ms for the forward product); in the even CTA warp 1 issues four M=256, N=256,
// K=16 MMAs per chunk under elect.sync into one of two TMEM accumulators (256
// columns each, in both CTAs) and warp 2 performs its mbarrier waits and meets
// it at a named-barrier rendezvous (a memory access of the issuing warp would
// wait behind its queued MMAs); warps 3-6 of each CTA drain their 128 rows of
// the previous item's accumulator to global memory meanwhile.  MMA completions
// reach both CTAs (commit to both); the epilogue warps release an accumulator
// on the even CTA's barrier.  All waits are bounded and both CTAs always reach
// the final cluster barrier.
#pragma once

#include "fna2_kernels.cuh"
#include "ptx.cuh"

namespace fna2 {

constexpr int kGemmBM = 256, kGemmBN = 256, kGemmBK = 64, kGemmStages = 6;  // BM, BN: per pair
constexpr int kGemmThreads = 224;           // producer, MMA issuer, waiter, 4 epilogue warps
constexpr uint32_t kGemmHandoffBar = 1;     // named barrier of the issuer / waiter rendezvous

struct GemmParams {
  int64_t M, N, K;
  int a_mn, b_mn;  // 1: operand stored MN-major
  void* c;
  int64_t ldc;
  int c_f32;       // 0: store bf16; 1: add fp32 partials (split over K)
  int chunks;      // 64-deep K chunks in total
  int chunks_per_split;
  int tiles_n, tiles;  // output tiles along N, in total
  int items;           // tiles x K slices
};

struct GemmSmem {
  static constexpr int kABytes = 128 * kGemmBK * 2;  // this CTA's 128 rows of A: 16 KB
  static constexpr int kBBytes = 128 * kGemmBK * 2;  // this CTA's 128 columns of B: 16 KB
  static constexpr int kStage = kABytes + kBBytes;
  static constexpr int oStaging = kGemmStages * kStage;  // 4 KB per epilogue warp
  static constexpr int oBar = oStaging + 4 * 4096;
  static constexpr int kNumBars = 2 * kGemmStages + 4;   // full, empty, acc_full[2], acc_empty[2]
  static constexpr int oMisc = oBar + kNumBars * 8;
  static constexpr int kTotal = oMisc + 16 + 1024;
  static_assert(kTotal <= kMaxDynamicSmem, "shared memory budget");
};

// Tile and chunk range of work item i (the same in every role of both CTAs).
__device__ __forceinline__ void gemm_item(const GemmParams& p, int i, int64_t& m0, int64_t& n0, int& c0, int& nc) {
  const int z = i / p.tiles, tile = i % p.tiles;
  n0 = static_cast<int64_t>(tile % p.tiles_n) * kGemmBN;
  m0 = static_cast<int64_t>(tile / p.tiles_n) * kGemmBM;
  c0 = z * p.chunks_per_split;
  nc = max(0, min(p.chunks, c0 + p.chunks_per_split) - c0);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    fna2_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const GemmParams p) {
  using L = GemmSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::oBar);
  uint64_t* full = bars;                     // even CTA: both CTAs' chunk landed
  uint64_t* empty = bars + kGemmStages;      // both CTAs: the chunk's MMAs are done
  uint64_t* acc_full = bars + 2 * kGemmStages;  // both CTAs
  uint64_t* acc_empty = acc_full + 2;           // even CTA: 4 epilogue warps x 2 CTAs
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::oMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::oMisc + 4);
  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cluster_ctarank();
  const int pair = static_cast<int>(blockIdx.x >> 1), n_pairs = static_cast<int>(gridDim.x >> 1);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised and the pair's TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto lead = [&](uint64_t* bar) { return mapa_shared(bar, 0); };

  if (warp == 0) {
    // ------------------------------------------------------------ producer (both CTAs)
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      int g = 0;  // chunks loaded so far (ring position)
      bool ok = true;
      for (int i = pair; ok && i < p.items; i += n_pairs) {
        int64_t m0, n0;
        int c0, nc;
        gemm_item(p, i, m0, n0, c0, nc);
        const int mr = static_cast<int>(m0) + 128 * static_cast<int>(rank);  // this CTA's rows of A
        const int nr = static_cast<int>(n0) + 128 * static_cast<int>(rank);  // this CTA's columns of the tile
        for (int c = 0; c < nc; ++c, ++g) {
          const int s = g % kGemmStages;
          if (g >= kGemmStages && !mbar_wait(&empty[s], ((g / kGemmStages) - 1) & 1, abort_flag, 1401)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * L::kStage;
          uint8_t* sb = sa + L::kABytes;
          const int k0 = (c0 + c) * kGemmBK;
          const uint32_t fb = lead(&full[s]);
          // the even CTA registers both CTAs' bytes with one local arrival; the odd
          // CTA's loads only complete bytes on that barrier (no remote arrival)
          if (rank == 0) mbar_expect_tx(&full[s], 2 * L::kStage);
          if (p.a_mn) {  // two 64-column (M) x 64-row (K) boxes
            for (int h = 0; h < 2; ++h) tma_load_4d_pair(sa + h * 8192, &tmA, fb, mr + 64 * h, k0, 0, 0);
          } else {  // one 64-column (K) x 128-row (M) box
            tma_load_4d_pair(sa, &tmA, fb, k0, mr, 0, 0);
          }
          if (p.b_mn) {
            for (int h = 0; h < 2; ++h) tma_load_4d_pair(sb + h * 8192, &tmB, fb, nr + 64 * h, k0, 0, 0);
          } else {
            tma_load_4d_pair(sb, &tmB, fb, k0, nr, 0, 0);
          }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    // The whole warp follows the hand-off sequence; an elected lane issues.
    if (rank == 0) {
      const uint32_t idesc = make_idesc_bf16(kGemmBM, kGemmBN, p.a_mn, p.b_mn);
      bool ok = true;
      int g = 0, it = 0;
      for (int i = pair; ok && i < p.items; i += n_pairs) {
        int64_t m0, n0;
        int c0, nc;
        gemm_item(p, i, m0, n0, c0, nc);
        if (nc == 0) continue;
        const int b = it & 1;
        const uint32_t tacc = tmem + 256 * b;
        for (int c = 0; c < nc; ++c, ++g) {
          // chunk g landed in both CTAs (and, for the first chunk, accumulator b drained)
          ok = pair_rendezvous(kGemmHandoffBar, ok);
          if (!ok) break;
          tc_fence_after();
          const int s = g % kGemmStages;
          const uint32_t sa = smem_u32(smem + s * L::kStage), sb = sa + L::kABytes;
          uint64_t ad[4], bd[4];
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            ad[kk] = p.a_mn ? make_sdesc(sa + kk * 2048, 8192, 1024, kSwizzle128B) : make_sdesc(sa + kk * 32, 16, 1024, kSwizzle128B);
            bd[kk] = p.b_mn ? make_sdesc(sb + kk * 2048, 8192, 1024, kSwizzle128B) : make_sdesc(sb + kk * 32, 16, 1024, kSwizzle128B);
          }
          if (elect_one()) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) mma_pair_ss(tacc, ad[kk], bd[kk], idesc, (c > 0 || kk > 0) ? 1u : 0u);
            mma_pair_commit_both(&empty[s]);
            if (c == nc - 1) mma_pair_commit_both(&acc_full[b]);
          }
          __syncwarp();
        }
        ++it;
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ waiter for the issuer (even CTA)
    if (rank == 0) {
      bool ok = true;
      int g = 0, it = 0;
      for (int i = pair; ok && i < p.items; i += n_pairs) {
        int64_t m0, n0;
        int c0, nc;
        gemm_item(p, i, m0, n0, c0, nc);
        if (nc == 0) continue;
        for (int c = 0; c < nc; ++c, ++g) {
          if (ok && c == 0 && it >= 2) ok = mbar_wait(&acc_empty[it & 1], ((it >> 1) - 1) & 1, abort_flag, 1404);
          if (ok) ok = mbar_wait(&full[g % kGemmStages], (g / kGemmStages) & 1, abort_flag, 1402);
          ok = pair_rendezvous(kGemmHandoffBar, ok);
          if (!ok) break;
        }
        ++it;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 3-6, both CTAs)
    const int q = warp & 3;  // TMEM lane quadrant = rows [32q, 32q+32) of this CTA's 128
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    uint8_t* stage = smem + L::oStaging + (warp - 3) * 4096;
    int it = 0;
    for (int i = pair; i < p.items; i += n_pairs) {
      int64_t m0, n0;
      int c0, nc;
      gemm_item(p, i, m0, n0, c0, nc);
      if (nc == 0) continue;
      const int b = it & 1;
      if (!mbar_wait(&acc_full[b], (it >> 1) & 1, abort_flag, 1403)) break;
      tc_fence_after();
      const int64_t row0 = m0 + 128 * rank + 32 * q;
      const int nvalid = static_cast<int>(p.M - row0 < 32 ? p.M - row0 : 32);
#pragma unroll 1
      for (int c = 0; c < kGemmBN / 32; ++c) {
        const int64_t col0 = n0 + 32 * c;
        if (col0 >= p.N) break;
        uint32_t v[32];
        tmem_ld32(tmem + 256 * b + lane_base + 32 * c, v);
        tmem_ld_wait32(v);
        if (!p.c_f32) {
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) pk[k] = pack_bf16(__uint_as_float(v[2 * k]), __uint_as_float(v[2 * k + 1]));
          if (nvalid > 0)
            warp_store_rows<16>(stage, pk, static_cast<__nv_bfloat16*>(p.c) + row0 * p.ldc + col0, p.ldc, nvalid);
        } else {
          // transpose through shared memory so that each reduction covers 128
          // contiguous bytes of one row (XOR swizzle: conflict-free both ways)
          float* st = reinterpret_cast<float*>(stage);
#pragma unroll
          for (int k = 0; k < 32; ++k) st[lane * 32 + (k ^ lane)] = __uint_as_float(v[k]);
          __syncwarp();
          float* crow = static_cast<float*>(p.c) + row0 * p.ldc + col0 + lane;
          for (int r = 0; r < nvalid; ++r) atomicAdd(crow + r * p.ldc, st[r * 32 + (lane ^ r)]);
          __syncwarp();
        }
      }
      // this CTA's half of accumulator b may take item it+2
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(lead(&acc_empty[b]));
      ++it;
    }
  }

  // Both CTAs: every MMA of the pair, every TMEM read and every cross-CTA
  // arrival is done before the pair's TMEM is released and either CTA exits.
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

inline cudaError_t launch_gemm(const CUtensorMap& a, const CUtensorMap& b, const GemmParams& p, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(fna2_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, GemmSmem::kTotal);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int pairs = p.items < sms / 2 ? p.items : sms / 2;
  fna2_gemm_kernel<<<2 * pairs, kGemmThreads, GemmSmem::kTotal, stream>>>(a, b, p);
  return cudaGetLastError();
}

}  // namespace fna2

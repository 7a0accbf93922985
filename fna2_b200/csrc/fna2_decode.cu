// KV-cache decode with the relational bias: one new query token per sequence
// attends to every cached key of its sequence (plus, optionally, its own new
// key, which the call appends to the caches).
//
// Logits follow the op's definition for the last query row of a sequence:
//   S[h,j] = scale * <q_h, k_j> + gs[h] * <r_q,h, r_k[j,h]>   (h <  H_G)
//   S[h,j] = scale * <q_h, k_j>                              (h >= H_G)
//   O = softmax(S) V,  O = acc/(l+1e-6),  LSE = m + log(l+1e-6)
// (FNA2/flash_naylis_attn.py:159-165,192,195; GQA kv head h / (H/H_KV), :99).
// The reference drops the bias at decode (FNA2/attention_fna2.py:428-432: the
// FNA2 path is bypassed when a KV cache is passed and graph_bias is skipped
// because R_k is not cached); this path caches R_k per graph head and keeps it.
//
// The work is HBM-bound (each cached key is read once per step).  One CTA
// serves (sequence, KV head, block of up to 16 query heads, key split); its 4
// warps stream their own 16-key tiles through per-warp rings of asynchronous
// copies and run the tiles on mma.sync m16n8k16 (bf16 in, fp32 out): rows are
// the query heads of the KV group, so one instruction covers the whole group
// and no bf16 unpacking or cross-lane reductions are needed per key.  The bias
// rides in the same instructions: the A operand is [q | R~_q] with
// R~_q = bf16(r_q * gs[h] / scale) placed block-diagonally (row h holds its own
// R~_q in the columns of head h's R_k), the B operand is [k_j | r_k[j, heads]],
// as the prefill kernels fold the bias.  Splits of one (sequence, head)
// combine in a second kernel.
#include "fna2_kernels.cuh"

namespace fna2 {

struct DecodeParams {
  int B, H, HKV, HG, R, G;  // G = H / HKV query heads per KV head
  int capacity;             // cache slots per sequence
  float scale, scale_log2;
  const __nv_bfloat16* q;
  int64_t q_sb, q_sh;
  const __nv_bfloat16* rq;
  int64_t rq_sb, rq_sh;
  __nv_bfloat16* kc;
  int64_t k_sb, k_st, k_sh;
  __nv_bfloat16* vc;
  int64_t v_sb, v_st, v_sh;
  __nv_bfloat16* rkc;
  int64_t rk_sb, rk_st, rk_sh;
  const float* gs;
  const int* seqlens;  // [B] keys already cached
  const int* offsets;  // optional [B]: first cache row of sequence b (packed caches)
  const __nv_bfloat16* kn;
  int64_t kn_sb, kn_sh;
  const __nv_bfloat16* vn;
  int64_t vn_sb, vn_sh;
  const __nv_bfloat16* rkn;
  int64_t rkn_sb, rkn_sh;
  __nv_bfloat16* out;
  int64_t o_sb, o_sh;
  float* lse;  // optional [B, H]
  float* ws;   // [B*H][splits][D + 2] partial (acc, m, l) when splits > 1
  int splits, head_blocks, stages;
};

constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecKeys = 16;  // keys per tile
constexpr int kDecodeStatusBadLength = 601;

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void dec_cp16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void dec_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void dec_wait(int pending) {
  // the ring depth is a launch parameter (2..4): pending = stages - 1
  if (pending >= 3)
    asm volatile("cp.async.wait_group 3;" ::: "memory");
  else if (pending == 2)
    asm volatile("cp.async.wait_group 2;" ::: "memory");
  else if (pending == 1)
    asm volatile("cp.async.wait_group 1;" ::: "memory");
  else
    asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Shared-memory geometry of one CTA (host and device agree on it).
struct DecodeSmem {
  int ke;        // extended key width: D + (graph heads of the block) * R
  int a_stride;  // bytes per row of [q | R~_q] (padded against ldmatrix bank conflicts)
  int k_stride;  // bytes per row of a [k | r_k] tile
  int v_stride;  // bytes per row of a V tile
  int stage;     // bytes per ring stage
  __host__ __device__ DecodeSmem(int D, int ng, int R) {
    ke = D + ng * R;
    a_stride = ke * 2 + 16;
    k_stride = a_stride;
    v_stride = D * 2 + 16;
    stage = kDecKeys * (k_stride + v_stride);
  }
  __host__ __device__ int a_bytes() const { return 16 * a_stride; }
  __host__ __device__ size_t total(int stages) const {
    const size_t ring = static_cast<size_t>(kDecWarps) * stages * stage;
    return a_bytes() + ring;
  }
};

template <int D>
__global__ void __launch_bounds__(kDecThreads) fna2_decode_kernel(const DecodeParams p) {
  extern __shared__ __align__(16) uint8_t dsm[];
  const int split = blockIdx.y;  // grid: x = (sequence, KV head, head block), y = key split (<= 64)
  const int hb = blockIdx.x % p.head_blocks;
  const int kh = (blockIdx.x / p.head_blocks) % p.HKV;
  const int b = blockIdx.x / (p.head_blocks * p.HKV);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h0 = kh * p.G + hb * 16;
  const int nh = min(16, p.G - hb * 16);
  const int ng = max(0, min(nh, p.HG - h0));  // graph heads in this block: h0 .. h0+ng-1
  const DecodeSmem L(D, ng, p.R);

  const int len0 = __ldg(p.seqlens + b);
  const bool has_new = p.kn != nullptr;
  const int len = len0 + (has_new ? 1 : 0);
  const bool bad = len0 < 0 || len > p.capacity;
  if (bad && threadIdx.x == 0 && split == 0 && blockIdx.x % (p.head_blocks * p.HKV) == 0) atomicCAS(&g_device_error, 0, kDecodeStatusBadLength);
  const int n_keys = bad ? 0 : len;
  const int per_split = ((n_keys + p.splits - 1) / p.splits + kDecKeys - 1) / kDecKeys * kDecKeys;
  const int k_begin = min(n_keys, split * per_split), k_end = min(n_keys, k_begin + per_split);
  const int64_t seq_row = p.offsets ? static_cast<int64_t>(__ldg(p.offsets + b)) : 0;

  // Append the new token's k, v (KV head kh, once per KV head) and r_k (graph heads of this block).
  if (has_new && !bad && len0 >= k_begin && len0 < k_end && warp == 0) {
    const int64_t row = seq_row + len0;
    if (hb == 0)
      for (int e = lane; e < D / 8; e += 32) {
        reinterpret_cast<uint4*>(p.kc + (p.offsets ? 0 : b * p.k_sb) + row * p.k_st + kh * p.k_sh)[e] =
            reinterpret_cast<const uint4*>(p.kn + b * p.kn_sb + kh * p.kn_sh)[e];
        reinterpret_cast<uint4*>(p.vc + (p.offsets ? 0 : b * p.v_sb) + row * p.v_st + kh * p.v_sh)[e] =
            reinterpret_cast<const uint4*>(p.vn + b * p.vn_sb + kh * p.vn_sh)[e];
      }
    for (int e = lane; e < ng * p.R / 8; e += 32) {
      const int g = e / (p.R / 8), c = e % (p.R / 8);
      reinterpret_cast<uint4*>(p.rkc + (p.offsets ? 0 : b * p.rk_sb) + row * p.rk_st + (h0 + g) * p.rk_sh)[c] =
          reinterpret_cast<const uint4*>(p.rkn + b * p.rkn_sb + (h0 + g) * p.rkn_sh)[c];
    }
  }

  // A = [q | R~_q] for the 16 rows (query heads h0..h0+15; rows past nh are zero).
  uint8_t* sa = dsm;
  for (int e = threadIdx.x; e < 16 * (L.ke / 8); e += kDecThreads) {
    const int row = e / (L.ke / 8), c8 = e % (L.ke / 8), col = c8 * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (row < nh) {
      const int h = h0 + row;
      if (col < D) {
        v = *reinterpret_cast<const uint4*>(p.q + b * p.q_sb + h * p.q_sh + col);
      } else {
        const int g = (col - D) / p.R, r0 = (col - D) % p.R;
        if (g == row) {  // block-diagonal: row h carries its own R~_q
          const float f = __ldg(p.gs + h) / p.scale;
          const uint4 w = *reinterpret_cast<const uint4*>(p.rq + b * p.rq_sb + h * p.rq_sh + r0);
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
          uint32_t o[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ww[i]));
            o[i] = pack_bf16(f2.x * f, f2.y * f);
          }
          v = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
    }
    *reinterpret_cast<uint4*>(sa + row * L.a_stride + col * 2) = v;
  }
  __syncthreads();

  // Per-warp ring of 16-key tiles: tile t of this warp covers keys k_begin + (warp + t*4) * 16.
  uint8_t* ring = dsm + L.a_bytes() + static_cast<size_t>(warp) * p.stages * L.stage;
  const int n_tiles_all = (k_end - k_begin + kDecKeys - 1) / kDecKeys;
  const int n_tiles = n_tiles_all > warp ? (n_tiles_all - warp + kDecWarps - 1) / kDecWarps : 0;
  const int kpieces = L.ke / 8, vpieces = D / 8;  // 16-byte pieces per row
  const int64_t kbase_b = p.offsets ? 0 : b * p.k_sb, vbase_b = p.offsets ? 0 : b * p.v_sb;
  const int64_t rbase_b = p.offsets ? 0 : b * p.rk_sb;
  // Whole tiles away from the appended slot take a fast path: each lane copies
  // fixed 16-byte pieces (column c of rows r0, r0 + RPP, ...) of K and V and
  // steps one pointer per pass; the tile holding the new token, and a partial
  // last tile, take the general path.
  constexpr int PPR = D / 8, RPP = 32 / PPR;  // pieces per K/V row, rows per pass
  const int pc = lane % PPR, pr0 = lane / PPR;
  const int rpieces = kpieces - PPR;          // R_k pieces per row (ng * R / 8)
  const int64_t kstep = static_cast<int64_t>(RPP) * p.k_st, vstep = static_cast<int64_t>(RPP) * p.v_st;
  const __nv_bfloat16* kcol = p.kc + kbase_b + seq_row * p.k_st + kh * p.k_sh + pc * 8;
  const __nv_bfloat16* vcol = p.vc + vbase_b + seq_row * p.v_st + kh * p.v_sh + pc * 8;
  int issued = 0;
  auto issue_general = [&](uint8_t* st, int j0) {
    for (int e = lane; e < kDecKeys * (kpieces + vpieces); e += 32) {
      const bool is_v = e >= kDecKeys * kpieces;
      const int ee = is_v ? e - kDecKeys * kpieces : e;
      const int np = is_v ? vpieces : kpieces;
      const int r = ee / np, c = ee % np, j = j0 + r;
      const bool valid = j < k_end;
      const bool fresh = has_new && j == len0;
      const int64_t row = seq_row + j;
      const __nv_bfloat16* src;
      if (is_v) {
        src = fresh ? p.vn + b * p.vn_sb + kh * p.vn_sh : p.vc + vbase_b + row * p.v_st + kh * p.v_sh;
        src += c * 8;
      } else if (c < D / 8) {
        src = fresh ? p.kn + b * p.kn_sb + kh * p.kn_sh : p.kc + kbase_b + row * p.k_st + kh * p.k_sh;
        src += c * 8;
      } else {
        const int g = (c - D / 8) / (p.R / 8), rc = (c - D / 8) % (p.R / 8);
        src = fresh ? p.rkn + b * p.rkn_sb + (h0 + g) * p.rkn_sh
                    : p.rkc + rbase_b + row * p.rk_st + (h0 + g) * p.rk_sh;
        src += rc * 8;
      }
      uint8_t* dst = is_v ? st + kDecKeys * L.k_stride + r * L.v_stride + c * 16 : st + r * L.k_stride + c * 16;
      dec_cp16(dst, valid ? static_cast<const void*>(src) : static_cast<const void*>(p.q), valid);
    }
  };
  auto issue = [&]() {
    if (issued < n_tiles) {
      uint8_t* st = ring + (issued % p.stages) * L.stage;
      const int j0 = k_begin + (warp + issued * kDecWarps) * kDecKeys;
      const bool whole = j0 + kDecKeys <= k_end && !(has_new && len0 >= j0 && len0 < j0 + kDecKeys);
      if (!whole) {
        issue_general(st, j0);
      } else {
        const __nv_bfloat16* ks = kcol + static_cast<int64_t>(j0 + pr0) * p.k_st;
        const __nv_bfloat16* vs = vcol + static_cast<int64_t>(j0 + pr0) * p.v_st;
        uint8_t* kd = st + pr0 * L.k_stride + pc * 16;
        uint8_t* vd = st + kDecKeys * L.k_stride + pr0 * L.v_stride + pc * 16;
#pragma unroll
        for (int i = 0; i < kDecKeys / RPP; ++i) {
          dec_cp16(kd + i * RPP * L.k_stride, ks + i * kstep, true);
          dec_cp16(vd + i * RPP * L.v_stride, vs + i * vstep, true);
        }
        for (int e = lane; e < kDecKeys * rpieces; e += 32) {  // R_k of the block's graph heads
          const int r = e / rpieces, c = e % rpieces;
          const int gh = c / (p.R / 8), rc = c % (p.R / 8);
          const __nv_bfloat16* src = p.rkc + rbase_b + (seq_row + j0 + r) * p.rk_st + (h0 + gh) * p.rk_sh + rc * 8;
          dec_cp16(st + r * L.k_stride + (PPR + c) * 16, src, true);
        }
      }
    }
    ++issued;
    dec_commit();
  };
  for (int s = 0; s < p.stages - 1; ++s) issue();

  const int g = lane >> 2, t = lane & 3;
  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // rows g and g+8 (log2 domain)
  const uint32_t a_addr = smem_u32(sa) + ((lane & 7) + ((lane >> 3) & 1) * 8) * L.a_stride + (lane >> 4) * 16;
  const float sl2 = p.scale_log2;

  for (int tt = 0; tt < n_tiles; ++tt) {
    __syncwarp();
    issue();
    dec_wait(p.stages - 1);
    __syncwarp();
    const uint8_t* st = ring + (tt % p.stages) * L.stage;
    const int j0 = k_begin + (warp + tt * kDecWarps) * kDecKeys;
    // S = [q | R~_q] [k | r_k]^T for 16 heads x 16 keys
    float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
    const uint32_t k_addr = smem_u32(st) + ((lane & 7) + (lane >> 4) * 8) * L.k_stride + ((lane >> 3) & 1) * 16;
    for (int ks = 0; ks < L.ke / 16; ++ks) {
      uint32_t a[4], kb[4];
      ldsm_x4(a, a_addr + ks * 32);
      ldsm_x4(kb, k_addr + ks * 32);
      mma_bf16(s0, a, kb[0], kb[1]);
      mma_bf16(s1, a, kb[2], kb[3]);
    }
    // online softmax on rows g (s[0], s[1]) and g+8 (s[2], s[3]); keys j0+2t, +1 (s0) and j0+8+2t, +1 (s1)
    float x[8] = {s0[0], s0[1], s1[0], s1[1], s0[2], s0[3], s1[2], s1[3]};
    const int kk[4] = {j0 + 2 * t, j0 + 2 * t + 1, j0 + 8 + 2 * t, j0 + 9 + 2 * t};
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = kk[i & 3] < k_end ? x[i] * sl2 : -INFINITY;
    float mx0 = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3])), mx1 = fmaxf(fmaxf(x[4], x[5]), fmaxf(x[6], x[7]));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    const float c0 = n0 == -INFINITY ? 1.f : exp2f(m0 - n0), c1 = n1 == -INFINITY ? 1.f : exp2f(m1 - n1);
    const float b0 = n0 == -INFINITY ? 0.f : n0, b1 = n1 == -INFINITY ? 0.f : n1;
#pragma unroll
    for (int i = 0; i < 4; ++i) x[i] = exp2f(x[i] - b0), x[4 + i] = exp2f(x[4 + i] - b1);
    l0 = l0 * c0 + (x[0] + x[1] + x[2] + x[3]);
    l1 = l1 * c1 + (x[4] + x[5] + x[6] + x[7]);
    m0 = n0, m1 = n1;
    if (__any_sync(0xffffffffu, c0 != 1.f || c1 != 1.f)) {  // no row max moved: the factors are exactly 1
#pragma unroll
      for (int i = 0; i < D / 8; ++i) acc[i][0] *= c0, acc[i][1] *= c0, acc[i][2] *= c1, acc[i][3] *= c1;
    }
    // O += P V: P (16 heads x 16 keys) is the A operand straight from the S fragments
    const uint32_t pa[4] = {pack_bf16(x[0], x[1]), pack_bf16(x[4], x[5]), pack_bf16(x[2], x[3]),
                            pack_bf16(x[6], x[7])};
    const uint32_t v_addr = smem_u32(st + kDecKeys * L.k_stride) +
                            ((lane & 7) + ((lane >> 3) & 1) * 8) * L.v_stride + (lane >> 4) * 16;
#pragma unroll
    for (int d16 = 0; d16 < D / 16; ++d16) {
      uint32_t vb[4];
      ldsm_x4_t(vb, v_addr + d16 * 32);
      mma_bf16(acc[2 * d16], pa, vb[0], vb[1]);
      mma_bf16(acc[2 * d16 + 1], pa, vb[2], vb[3]);
    }
  }
  dec_wait(0);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  // Combine the 4 warps through shared memory (the rings are done).
  __syncthreads();
  float* cm = reinterpret_cast<float*>(dsm);                 // [warps][16] m
  float* cl = cm + kDecWarps * 16;                            // [warps][16] l
  float* co = cl + kDecWarps * 16;                            // [warps][16][D] acc
  if (t == 0) {
    cm[warp * 16 + g] = m0, cm[warp * 16 + g + 8] = m1;
    cl[warp * 16 + g] = l0, cl[warp * 16 + g + 8] = l1;
  }
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    float* r0 = co + (warp * 16 + g) * D + i * 8 + 2 * t;
    float* r1 = co + (warp * 16 + g + 8) * D + i * 8 + 2 * t;
    r0[0] = acc[i][0], r0[1] = acc[i][1], r1[0] = acc[i][2], r1[1] = acc[i][3];
  }
  __syncthreads();
  for (int e = threadIdx.x; e < nh * D; e += kDecThreads) {
    const int row = e / D, d = e % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, cm[w * 16 + row]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kDecWarps; ++w) {
        const float f = exp2f(cm[w * 16 + row] - M);
        Ls += cl[w * 16 + row] * f;
        O += co[(w * 16 + row) * D + d] * f;
      }
    }
    const int h = h0 + row;
    if (p.splits == 1) {
      p.out[b * p.o_sb + h * p.o_sh + d] = __float2bfloat16_rn(O / (Ls + 1e-6f));
      if (d == 0 && p.lse) p.lse[b * p.H + h] = M * 0.69314718055994531f + logf(Ls + 1e-6f);
    } else {
      float* w = p.ws + ((static_cast<int64_t>(b) * p.H + h) * p.splits + split) * (D + 2);
      w[d] = O;
      if (d == 0) w[D] = M, w[D + 1] = Ls;
    }
  }
}

// Merge the splits of one (sequence, query head): rescale to the common max,
// then O = acc / (l + 1e-6), LSE = m + log(l + 1e-6) (natural log).
template <int D>
__global__ void __launch_bounds__(D) fna2_decode_combine_kernel(const DecodeParams p) {
  const int bh = blockIdx.x, b = bh / p.H, h = bh % p.H, d = threadIdx.x;
  const float* w = p.ws + static_cast<int64_t>(bh) * p.splits * (D + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, w[s * (D + 2) + D]);
  float Ls = 0.f, O = 0.f;
  if (M != -INFINITY)
    for (int s = 0; s < p.splits; ++s) {
      const float f = exp2f(w[s * (D + 2) + D] - M);
      Ls += w[s * (D + 2) + D + 1] * f;
      O += w[s * (D + 2) + d] * f;
    }
  p.out[b * p.o_sb + h * p.o_sh + d] = __float2bfloat16_rn(O / (Ls + 1e-6f));
  if (d == 0 && p.lse) p.lse[b * p.H + h] = M * 0.69314718055994531f + logf(Ls + 1e-6f);
}

// Ring depth that keeps a CTA at or under ~100 KB of shared memory (two CTAs
// per SM), between 2 and 4 stages.
inline int decode_stages(int D, int ng_max, int R) {
  const DecodeSmem L(D, ng_max, R);
  for (int s = 4; s > 2; --s)
    if (L.total(s) <= 100 * 1024) return s;
  return 2;
}

inline size_t decode_smem_bytes(int D, int ng_max, int R, int stages) {
  const DecodeSmem L(D, ng_max, R);
  const size_t combine = static_cast<size_t>(kDecWarps) * 16 * (D + 2) * 4;
  return std::max(L.total(stages), combine);
}

template <int D>
cudaError_t launch_decode_t(const DecodeParams& p, size_t smem, cudaStream_t stream) {
  auto kern = fna2_decode_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  const dim3 grid(p.B * p.HKV * p.head_blocks, p.splits);
  kern<<<grid, kDecThreads, smem, stream>>>(p);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  if (p.splits > 1) {
    fna2_decode_combine_kernel<D><<<p.B * p.H, D, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  return e;
}

inline cudaError_t launch_decode(const DecodeParams& p, int D, size_t smem, cudaStream_t stream) {
  if (D == 128) return launch_decode_t<128>(p, smem, stream);
  if (D == 64) return launch_decode_t<64>(p, smem, stream);
  return cudaErrorInvalidValue;
}

}  // namespace fna2

// Varlen QK-RMSNorm + RoPE pre-attention transform (forward and backward).
//
// Reference semantics: FNA2/attention_fna2.py RMSNorm.forward (:100-102):
// n = x * rsqrt(mean(x^2) + eps) * w; RotaryPositionalEmbedding (:108-163):
// y = n*cos + rotate_half(n)*sin with cos/sin = cos/sin(cat(t*f, t*f)), the
// table built in the dtype of the rotated tensor (:148-155); and
// _apply_rope_varlen (:620-647): t restarts at 0 for every packed sequence.
//
// HBM-bound elementwise work.  Each warp owns a contiguous run of tokens and
// streams the rows (token, head) of that run through a small ring of
// asynchronous copies in shared memory.  A token's position comes from a
// warp-wide search over cu_seqlens (skipped while the run stays inside one
// sequence) and its cos/sin values are computed once and reused for all of its
// heads.  The backward recomputes the norm and reduces the weight gradients
// per warp, then per CTA, then with one atomic per column and CTA.
#include "fna2_kernels.cuh"

namespace fna2 {

struct QkRows {
  void* ptr;
  int64_t ts, hs;  // token, head strides (elements)
};

struct QkPrepParams {
  int64_t T;
  int N;
  const int* cu;
  int hq, hk;
  int in_bf16, w_bf16, rope_bf16;
  QkRows qi, ki, qo, ko;            // inputs (in dtype), outputs (bf16)
  QkRows dqo, dko, dqi, dki;        // backward: grads of outputs (bf16), grads of inputs (in dtype)
  const void* qw;
  const void* kw;
  float eps;
  const float* inv_freq;
  float* dqw;
  float* dkw;
};

constexpr int kPrepThreads = 256;

// Field-wise select of one of two row descriptors.  Selecting a reference to a
// kernel parameter at run time would make the compiler copy the parameters to
// local memory.
__device__ __forceinline__ QkRows pick(bool first, const QkRows& a, const QkRows& b) {
  QkRows r;
  r.ptr = first ? a.ptr : b.ptr;
  r.ts = first ? a.ts : b.ts;
  r.hs = first ? a.hs : b.hs;
  return r;
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Layout.  Rows move between HBM and shared memory as whole rows: piece i
// (16 bytes) of a unit of RB rows is copied by lane i % 32, so each warp
// instruction covers whole rows (instructions that cover half rows, 128 bytes
// apart, measured at two thirds of the bandwidth).  For the arithmetic a row
// is spread over LPR = D/16 lanes: lane `sub` of a row holds the 8 values
// [8*sub, 8*sub+8) of the first half and the 8 values [D/2 + 8*sub, ...) of
// the second half, so the rotate_half pairs (e, e + D/2) sit in one lane and
// RoPE needs no shuffles; row sums reduce over the row's LPR lanes.  A warp
// covers RPW = 32/LPR rows per row batch.
constexpr int kHPL = 8;         // values per lane per half row
constexpr int kPrepStages = 4;  // units in flight per warp

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Address of global row rr (< hq: a query head of A, else a key head of B) of token t.
template <int ES>
__device__ __forceinline__ uint8_t* row_addr(const QkPrepParams& p, const QkRows& A, const QkRows& B, int64_t t,
                                             int rr) {
  const bool isq = rr < p.hq;
  const QkRows m = pick(isq, A, B);
  return static_cast<uint8_t*>(m.ptr) + (t * m.ts + static_cast<int64_t>(isq ? rr : rr - p.hq) * m.hs) * ES;
}

// First byte of this lane's first piece when global rows [row0, row0 + RB) of
// token t all belong to one tensor (A: rows < hq, B: the rest) and all exist;
// nullptr otherwise.  *step: bytes between a lane's consecutive pieces.
template <int D, int RB, int ES>
__device__ __forceinline__ uint8_t* unit_rows(const QkPrepParams& p, const QkRows& A, const QkRows& B, int64_t t,
                                              int row0, int lane, int64_t* step) {
  constexpr int PPR = D * ES / 16;  // 16-byte pieces per row (8, 16 or 32)
  const bool in_a = row0 + RB <= p.hq, in_b = row0 >= p.hq && row0 + RB <= p.hq + p.hk;
  if (!in_a && !in_b) return nullptr;
  const QkRows m = pick(in_a, A, B);
  *step = (32 / PPR) * m.hs * ES;
  return static_cast<uint8_t*>(m.ptr) + (t * m.ts + static_cast<int64_t>(in_a ? row0 : row0 - p.hq) * m.hs) * ES +
         (lane / PPR) * m.hs * ES + (lane % PPR) * 16;
}

// Copy global rows [row0, row0 + RB) of token t into a row-major block at dst
// (rows past hq + hk are zero-filled).
template <int D, int RB, int ES>
__device__ __forceinline__ void stage_rows(uint8_t* dst, const QkPrepParams& p, const QkRows& A, const QkRows& B,
                                           int64_t t, int row0, int lane) {
  constexpr int PPR = D * ES / 16;
  static_assert((RB * PPR) % 32 == 0 && PPR <= 32, "a unit is whole warp instructions");
  int64_t step = 0;
  if (const uint8_t* g = unit_rows<D, RB, ES>(p, A, B, t, row0, lane, &step)) {
#pragma unroll
    for (int i = 0; i < RB * PPR / 32; ++i) cp_async16(dst + (i * 32 + lane) * 16, g + i * step, true);
    return;
  }
#pragma unroll
  for (int i = 0; i < RB * PPR / 32; ++i) {
    const int q = i * 32 + lane, rr = row0 + q / PPR;
    const bool valid = rr < p.hq + p.hk;
    const uint8_t* g = valid ? row_addr<ES>(p, A, B, t, rr) + (q % PPR) * 16 : static_cast<const uint8_t*>(A.ptr);
    cp_async16(dst + q * 16, g, valid);
  }
}

// Store the row-major block at src as global rows [row0, row0 + RB) of token t.
template <int D, int RB, int ES>
__device__ __forceinline__ void store_rows(const uint8_t* src, const QkPrepParams& p, const QkRows& A,
                                           const QkRows& B, int64_t t, int row0, int lane) {
  constexpr int PPR = D * ES / 16;
  int64_t step = 0;
  if (uint8_t* g = unit_rows<D, RB, ES>(p, A, B, t, row0, lane, &step)) {
#pragma unroll
    for (int i = 0; i < RB * PPR / 32; ++i)
      *reinterpret_cast<uint4*>(g + i * step) = *reinterpret_cast<const uint4*>(src + (i * 32 + lane) * 16);
    return;
  }
#pragma unroll
  for (int i = 0; i < RB * PPR / 32; ++i) {
    const int q = i * 32 + lane, rr = row0 + q / PPR;
    if (rr < p.hq + p.hk)
      *reinterpret_cast<uint4*>(row_addr<ES>(p, A, B, t, rr) + (q % PPR) * 16) =
          *reinterpret_cast<const uint4*>(src + q * 16);
  }
}

// 8 consecutive values (bf16 or fp32) from shared memory.
template <int ES>
__device__ __forceinline__ void lds8(const uint8_t* src, float (&x)[kHPL]) {
  if (ES == 2) {
    const uint4 w = *reinterpret_cast<const uint4*>(src);
    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ww[i]));
      x[2 * i] = f.x, x[2 * i + 1] = f.y;
    }
  } else {
    const float4 a = reinterpret_cast<const float4*>(src)[0], b = reinterpret_cast<const float4*>(src)[1];
    x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
  }
}

template <int ES>
__device__ __forceinline__ void sts8(uint8_t* dst, const float (&y)[kHPL]) {
  if (ES == 2) {
    *reinterpret_cast<uint4*>(dst) =
        make_uint4(pack_bf16(y[0], y[1]), pack_bf16(y[2], y[3]), pack_bf16(y[4], y[5]), pack_bf16(y[6], y[7]));
  } else {
    reinterpret_cast<float4*>(dst)[0] = make_float4(y[0], y[1], y[2], y[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(y[4], y[5], y[6], y[7]);
  }
}

// Sequence bounds [*lo, *hi) of token t (all lanes of the warp call it with the
// same t); returns false if t belongs to no sequence.  A 32-way search: each
// round the lanes probe 32 evenly spaced cu_seqlens entries.
__device__ __forceinline__ bool warp_find_sequence(const QkPrepParams& p, int64_t t, int lane, int* lo_out,
                                                   int* hi_out) {
  if (t < __ldg(p.cu) || t >= __ldg(p.cu + p.N)) return false;
  int lo = 0, hi = p.N;  // cu[lo] <= t < cu[hi]
  while (hi - lo > 1) {
    const int step = (hi - lo + 31) / 32;
    const int idx = min(lo + lane * step, hi);
    const bool le = idx < hi && __ldg(p.cu + idx) <= t;
    const unsigned m = __ballot_sync(0xffffffffu, le);
    const int last = 31 - __clz(m);  // lane 0 always qualifies
    lo = lo + last * step;
    hi = min(lo + step, hi);
  }
  *lo_out = __ldg(p.cu + lo);
  *hi_out = __ldg(p.cu + lo + 1);
  return true;
}

// cos/sin of this lane's 8 frequencies at position pos, formed as the reference
// forms its table: fp32 t*f, or (bf16 mode) t, f and t*f rounded to bf16 and
// cos/sin rounded to bf16.  The RPW row groups of a warp need the same values,
// so each lane evaluates VPL = 8/RPW of them (frequencies fr, preloaded) and
// the warp exchanges them; all lanes must call this together.
template <int LPR, int VPL>
__device__ __forceinline__ void rope_table(bool bf16_mode, int pos, int sub, const float (&fr)[VPL],
                                           float (&c)[kHPL], float (&s)[kHPL]) {
  float cm[VPL], sm[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const float t = static_cast<float>(pos);
    const float ang = bf16_mode ? bf16_round(bf16_round(t) * bf16_round(fr[i])) : t * fr[i];
    sincosf(ang, &sm[i], &cm[i]);
    if (bf16_mode) {
      cm[i] = bf16_round(cm[i]);
      sm[i] = bf16_round(sm[i]);
    }
  }
#pragma unroll
  for (int v = 0; v < kHPL; ++v) {  // entry v of this lane's columns sits in row group v / VPL
    c[v] = __shfl_sync(0xffffffffu, cm[v % VPL], (v / VPL) * LPR + sub);
    s[v] = __shfl_sync(0xffffffffu, sm[v % VPL], (v / VPL) * LPR + sub);
  }
}

__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 h) { return *reinterpret_cast<const uint32_t*>(&h); }

// y1 = x1*c + (-x2)*s and y2 = x2*c + x1*s on bf16 operands with the reference's
// roundings (each product rounded to bf16, then the sum), written as packed
// bf16 words.  Each bf16 product is exact in fp32 and a sum of two bf16 values
// rounds to the same bf16 whether or not it passes through fp32 first, so
// bf16x2 arithmetic reproduces the reference's fp32-computed bf16 ops.
__device__ __forceinline__ void rope_bf16_packed(const float (&x1)[kHPL], const float (&x2)[kHPL],
                                                 const float (&c)[kHPL], const float (&s)[kHPL], uint4& y1,
                                                 uint4& y2) {
  uint32_t o1[4], o2[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(x1[2 * i], x1[2 * i + 1]);
    const __nv_bfloat162 b = __floats2bfloat162_rn(x2[2 * i], x2[2 * i + 1]);
    const __nv_bfloat162 cc = __floats2bfloat162_rn(c[2 * i], c[2 * i + 1]);
    const __nv_bfloat162 sn = __floats2bfloat162_rn(s[2 * i], s[2 * i + 1]);
    o1[i] = bf162_bits(__hsub2(__hmul2_rn(a, cc), __hmul2_rn(b, sn)));
    o2[i] = bf162_bits(__hadd2(__hmul2_rn(b, cc), __hmul2_rn(a, sn)));
  }
  y1 = make_uint4(o1[0], o1[1], o1[2], o1[3]);
  y2 = make_uint4(o2[0], o2[1], o2[2], o2[3]);
}

// RMSNorm weights in shared memory are stored so that the lanes of a row read
// 16 consecutive bytes each (no bank conflicts): column e of half h sits in
// float4 slot (h * 2 + (e % 8) / 4) * LPR + e / 8, component e % 4.
template <int D>
__device__ __forceinline__ int w_slot(int col) {
  constexpr int LPR = D / (2 * kHPL);
  const int h = col / (D / 2), e = col % (D / 2);
  return ((h * 2 + (e % kHPL) / 4) * LPR + e / kHPL) * 4 + e % 4;
}

template <int D>
__device__ __forceinline__ void load_w(const float* sw, int sub, float (&w1)[kHPL], float (&w2)[kHPL]) {
  constexpr int LPR = D / (2 * kHPL);
  const float4* w4 = reinterpret_cast<const float4*>(sw);
  const float4 a = w4[sub], b = w4[LPR + sub], c = w4[2 * LPR + sub], d = w4[3 * LPR + sub];
  w1[0] = a.x, w1[1] = a.y, w1[2] = a.z, w1[3] = a.w, w1[4] = b.x, w1[5] = b.y, w1[6] = b.z, w1[7] = b.w;
  w2[0] = c.x, w2[1] = c.y, w2[2] = c.z, w2[3] = c.w, w2[4] = d.x, w2[5] = d.y, w2[6] = d.z, w2[7] = d.w;
}

template <int LPR, int N>
__device__ __forceinline__ void row_sums(float (&v)[N]) {
#pragma unroll
  for (int o = LPR / 2; o > 0; o >>= 1)
#pragma unroll
    for (int j = 0; j < N; ++j) v[j] += __shfl_xor_sync(0xffffffffu, v[j], o);
}

// Rows per streamed unit and the unit's bytes: operand 0 (x, or dy for the
// backward, bf16) then operand 1 (the backward's x).
constexpr int qk_unit_rows(int D, bool bwd, int eb) { return (bwd || eb == 4 ? 1 : 2) * (32 / (D / (2 * kHPL))); }
constexpr int qk_unit_bytes(int D, bool bwd, int eb) {
  return qk_unit_rows(D, bwd, eb) * D * (bwd ? 2 + eb : eb);
}

// Shared memory: the two RMSNorm weights (fp32), then the units of each warp's ring.
constexpr size_t qk_prep_smem(int D, bool bwd, int eb) {
  return static_cast<size_t>(2 * D * 4) + static_cast<size_t>(kPrepThreads / 32) * kPrepStages * qk_unit_bytes(D, bwd, eb);
}

// One kernel for both directions: BWD reads x and dy and writes dx (+ weight
// gradients); the forward reads x and writes y.  EB: bytes per input element.
template <int D, bool BWD, int EB>
__global__ void __launch_bounds__(kPrepThreads, BWD ? 2 : 3) fna2_qk_prep_kernel(const QkPrepParams p) {
  constexpr int LPR = D / (2 * kHPL), RPW = 32 / LPR;
  constexpr int RB = qk_unit_rows(D, BWD, EB), RBATCH = RB / RPW;  // rows, row batches per unit
  constexpr int E0 = BWD ? 2 : EB;                                  // bytes per element of operand 0
  constexpr int B0 = RB * D * E0, UNIT = qk_unit_bytes(D, BWD, EB);
  extern __shared__ __align__(16) uint8_t prep_smem[];
  float* s_w = reinterpret_cast<float*>(prep_smem);  // [2][D], columns placed by w_slot
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sub = lane % LPR, rsel = lane / LPR;
  const bool rope = p.inv_freq != nullptr, norm = p.qw != nullptr;
  const int rows = p.hq + p.hk, units_per_token = (rows + RB - 1) / RB;
  uint8_t* wbuf = prep_smem + 2 * D * 4 + static_cast<size_t>(warp) * kPrepStages * UNIT;
  if (norm)
    for (int e = threadIdx.x; e < 2 * D; e += kPrepThreads) {
      const void* w = e < D ? p.qw : p.kw;
      const int i = e % D;
      s_w[(e / D) * D + w_slot<D>(i)] = p.w_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(w)[i]) : static_cast<const float*>(w)[i];
    }
  __syncthreads();
  float gq1[kHPL], gq2[kHPL], gk1[kHPL], gk2[kHPL];  // weight gradients (backward)
#pragma unroll
  for (int v = 0; v < kHPL; ++v) gq1[v] = gq2[v] = gk1[v] = gk2[v] = 0.f;

  const int64_t nw = static_cast<int64_t>(gridDim.x) * (kPrepThreads / 32);
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * (kPrepThreads / 32) + warp;
  const int64_t chunk = (p.T + nw - 1) / nw;
  const int64_t run_beg = gw * chunk, run_end = min(p.T, run_beg + chunk);
  const int64_t n_units = run_end > run_beg ? (run_end - run_beg) * units_per_token : 0;
  // cursors (token, unit within the token) of the next unit to stage and to consume
  int64_t issue_n = 0, issue_t = run_beg, use_t = run_beg;
  int issue_b = 0, use_b = 0;
  auto issue = [&]() {
    if (issue_n < n_units) {
      uint8_t* st = wbuf + (issue_n % kPrepStages) * UNIT;
      if (BWD) {
        stage_rows<D, RB, 2>(st, p, p.dqo, p.dko, issue_t, issue_b * RB, lane);
        if (norm) stage_rows<D, RB, EB>(st + B0, p, p.qi, p.ki, issue_t, issue_b * RB, lane);
      } else {
        stage_rows<D, RB, EB>(st, p, p.qi, p.ki, issue_t, issue_b * RB, lane);
      }
      if (++issue_b == units_per_token) issue_b = 0, ++issue_t;
      ++issue_n;
    }
    cp_async_commit();
  };
#pragma unroll
  for (int u = 0; u < kPrepStages - 1; ++u) issue();
  int s_lo = 0, s_hi = 0;
  bool inside = true;
  float c[kHPL], s[kHPL];
  constexpr int VPL = kHPL / RPW;
  float fr[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) fr[i] = rope ? __ldg(p.inv_freq + kHPL * sub + rsel * VPL + i) : 0.f;
  for (int64_t u = 0; u < n_units; ++u) {
    __syncwarp();  // every lane is done with the slot that this issue refills
    issue();
    cp_async_wait<kPrepStages - 1>();  // this lane's pieces of unit u have landed
    __syncwarp();                      // and so have the other lanes'
    const int64_t t = use_t;
    const int b = use_b;
    if (++use_b == units_per_token) use_b = 0, ++use_t;
    if (b == 0 && rope) {  // a new token: its position and cos/sin
      if (t < s_lo || t >= s_hi) {
        inside = warp_find_sequence(p, t, lane, &s_lo, &s_hi);
        if (!inside) s_lo = s_hi = 0;
      }
      if (inside) rope_table<LPR, VPL>(p.rope_bf16, static_cast<int>(t - s_lo), sub, fr, c, s);
    }
    uint8_t* st = wbuf + (u % kPrepStages) * UNIT;
    if (!BWD) {
      if (rope && !inside) continue;  // outside every sequence: left unset, as the reference does
      float x1[RBATCH][kHPL], x2[RBATCH][kHPL], ss[RBATCH];
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) {
        const uint8_t* rp = st + (j * RPW + rsel) * D * EB;
        lds8<EB>(rp + kHPL * sub * EB, x1[j]);
        lds8<EB>(rp + (D / 2 + kHPL * sub) * EB, x2[j]);
      }
      if (norm) {
#pragma unroll
        for (int j = 0; j < RBATCH; ++j) {
          ss[j] = 0.f;
#pragma unroll
          for (int v = 0; v < kHPL; ++v) ss[j] = fmaf(x1[j][v], x1[j][v], fmaf(x2[j][v], x2[j][v], ss[j]));
        }
        row_sums<LPR>(ss);
      }
      if (EB != 2) __syncwarp();  // the bf16 output rows overlap other lanes' fp32 input pieces
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) {
        const bool isq = b * RB + j * RPW + rsel < p.hq;
        if (norm) {
          const float rho = rsqrtf(ss[j] * (1.f / D) + p.eps);
          float w1[kHPL], w2[kHPL];
          load_w<D>(s_w + (isq ? 0 : D), sub, w1, w2);
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {
            x1[j][v] = x1[j][v] * rho * w1[v];
            x2[j][v] = x2[j][v] * rho * w2[v];
          }
        }
        uint8_t* op = st + (j * RPW + rsel) * D * 2;
        if (rope && p.rope_bf16) {
          uint4 y1, y2;
          rope_bf16_packed(x1[j], x2[j], c, s, y1, y2);
          *reinterpret_cast<uint4*>(op + kHPL * sub * 2) = y1;
          *reinterpret_cast<uint4*>(op + (D / 2 + kHPL * sub) * 2) = y2;
          continue;
        }
        if (rope) {
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {  // fp32: y1 = x1 c + (-x2) s, y2 = x2 c + x1 s, uncontracted
            const float a = x1[j][v], bb = x2[j][v];
            x1[j][v] = __fadd_rn(__fmul_rn(a, c[v]), -__fmul_rn(bb, s[v]));
            x2[j][v] = __fadd_rn(__fmul_rn(bb, c[v]), __fmul_rn(a, s[v]));
          }
        }
        sts8<2>(op + kHPL * sub * 2, x1[j]);
        sts8<2>(op + (D / 2 + kHPL * sub) * 2, x2[j]);
      }
      __syncwarp();
      store_rows<D, RB, 2>(st, p, p.qo, p.ko, t, b * RB, lane);
    } else {
      const bool zero = rope && !inside;  // outside every sequence: no path to the output
      float g1[RBATCH][kHPL], g2[RBATCH][kHPL], x1[RBATCH][kHPL], x2[RBATCH][kHPL];
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) {
        const uint8_t* gp = st + (j * RPW + rsel) * D * 2;
        lds8<2>(gp + kHPL * sub * 2, g1[j]);
        lds8<2>(gp + (D / 2 + kHPL * sub) * 2, g2[j]);
        if (norm) {
          const uint8_t* xp = st + B0 + (j * RPW + rsel) * D * EB;
          lds8<EB>(xp + kHPL * sub * EB, x1[j]);
          lds8<EB>(xp + (D / 2 + kHPL * sub) * EB, x2[j]);
        }
      }
      if (rope && !zero) {
#pragma unroll
        for (int j = 0; j < RBATCH; ++j)
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {  // transpose: dn1 = g1 c + g2 s, dn2 = g2 c - g1 s
            const float a = g1[j][v], bb = g2[j][v];
            g1[j][v] = a * c[v] + bb * s[v];
            g2[j][v] = bb * c[v] - a * s[v];
          }
      }
      if (norm && !zero) {
        float ss[RBATCH], dot[RBATCH];
#pragma unroll
        for (int j = 0; j < RBATCH; ++j) {
          const bool isq = b * RB + j * RPW + rsel < p.hq;
          float w1[kHPL], w2[kHPL];
          load_w<D>(s_w + (isq ? 0 : D), sub, w1, w2);
          ss[j] = dot[j] = 0.f;
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {
            ss[j] = fmaf(x1[j][v], x1[j][v], fmaf(x2[j][v], x2[j][v], ss[j]));
            dot[j] = fmaf(g1[j][v] * w1[v], x1[j][v], fmaf(g2[j][v] * w2[v], x2[j][v], dot[j]));
          }
        }
        row_sums<LPR>(ss);
        row_sums<LPR>(dot);
#pragma unroll
        for (int j = 0; j < RBATCH; ++j) {
          const int r = b * RB + j * RPW + rsel;
          const bool isq = r < p.hq;
          float w1[kHPL], w2[kHPL];
          load_w<D>(s_w + (isq ? 0 : D), sub, w1, w2);
          const float rho = rsqrtf(ss[j] * (1.f / D) + p.eps);
          const float k3 = dot[j] * rho * rho * rho * (1.f / D);
#pragma unroll
          for (int v = 0; v < kHPL; ++v) {
            if (r < rows) {
              if (isq) {
                gq1[v] = fmaf(g1[j][v], x1[j][v] * rho, gq1[v]);
                gq2[v] = fmaf(g2[j][v], x2[j][v] * rho, gq2[v]);
              } else {
                gk1[v] = fmaf(g1[j][v], x1[j][v] * rho, gk1[v]);
                gk2[v] = fmaf(g2[j][v], x2[j][v] * rho, gk2[v]);
              }
            }
            g1[j][v] = g1[j][v] * w1[v] * rho - x1[j][v] * k3;
            g2[j][v] = g2[j][v] * w2[v] * rho - x2[j][v] * k3;
          }
        }
      }
      // dx goes where this lane read its x pieces (operand 1, same element size)
#pragma unroll
      for (int j = 0; j < RBATCH; ++j) {
        if (zero) {
#pragma unroll
          for (int v = 0; v < kHPL; ++v) g1[j][v] = g2[j][v] = 0.f;
        }
        uint8_t* xp = st + B0 + (j * RPW + rsel) * D * EB;
        sts8<EB>(xp + kHPL * sub * EB, g1[j]);
        sts8<EB>(xp + (D / 2 + kHPL * sub) * EB, g2[j]);
      }
      __syncwarp();
      store_rows<D, RB, EB>(st + B0, p, p.dqi, p.dki, t, b * RB, lane);
    }
  }
  cp_async_wait<0>();
  if (BWD && norm) {
    // weight gradients: lanes of the same column positions, warps, CTA -> one atomic per column
#pragma unroll
    for (int o = LPR; o < 32; o <<= 1)
#pragma unroll
      for (int v = 0; v < kHPL; ++v) {
        gq1[v] += __shfl_xor_sync(0xffffffffu, gq1[v], o);
        gq2[v] += __shfl_xor_sync(0xffffffffu, gq2[v], o);
        gk1[v] += __shfl_xor_sync(0xffffffffu, gk1[v], o);
        gk2[v] += __shfl_xor_sync(0xffffffffu, gk2[v], o);
      }
    __syncthreads();  // the staging ring is reused as the reduction buffer
    float* s_dw = reinterpret_cast<float*>(prep_smem + 2 * D * 4);  // [warps][2][D]
    if (rsel == 0) {
#pragma unroll
      for (int v = 0; v < kHPL; ++v) {
        s_dw[(warp * 2 + 0) * D + kHPL * sub + v] = gq1[v];
        s_dw[(warp * 2 + 0) * D + D / 2 + kHPL * sub + v] = gq2[v];
        s_dw[(warp * 2 + 1) * D + kHPL * sub + v] = gk1[v];
        s_dw[(warp * 2 + 1) * D + D / 2 + kHPL * sub + v] = gk2[v];
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < 2 * D; e += kPrepThreads) {
      const int which = e / D, col = e % D;
      float acc = 0.f;
#pragma unroll
      for (int w8 = 0; w8 < kPrepThreads / 32; ++w8) acc += s_dw[(w8 * 2 + which) * D + col];
      atomicAdd((which ? p.dkw : p.dqw) + col, acc);
    }
  }
}

template <int D, bool BWD, int EB>
cudaError_t launch_qk_prep_t(const QkPrepParams& p, cudaStream_t stream) {
  auto kern = fna2_qk_prep_kernel<D, BWD, EB>;
  constexpr size_t smem = qk_prep_smem(D, BWD, EB);
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148, per_sm = 1;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPrepThreads, smem);
  if (e != cudaSuccess) return e;
  // one wave of resident CTAs, each warp at least 8 tokens
  const int64_t blocks = ((p.T + 7) / 8 + kPrepThreads / 32 - 1) / (kPrepThreads / 32);
  const int64_t wave = static_cast<int64_t>(sms) * (per_sm > 0 ? per_sm : 1);
  const int grid = static_cast<int>(blocks < wave ? (blocks > 0 ? blocks : 1) : wave);
  kern<<<grid, kPrepThreads, smem, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_qk_prep(const QkPrepParams& p, int D, bool bwd, cudaStream_t stream) {
  const bool b16 = p.in_bf16 != 0;
  if (D == 128) {
    if (bwd) return b16 ? launch_qk_prep_t<128, true, 2>(p, stream) : launch_qk_prep_t<128, true, 4>(p, stream);
    return b16 ? launch_qk_prep_t<128, false, 2>(p, stream) : launch_qk_prep_t<128, false, 4>(p, stream);
  }
  if (D == 64) {
    if (bwd) return b16 ? launch_qk_prep_t<64, true, 2>(p, stream) : launch_qk_prep_t<64, true, 4>(p, stream);
    return b16 ? launch_qk_prep_t<64, false, 2>(p, stream) : launch_qk_prep_t<64, false, 4>(p, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace fna2

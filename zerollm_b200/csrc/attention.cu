// attention.cu -- causal multi-head attention for the training step.
//
// bf16 path (the model): fused flash-style forward and backward over a
// packed qkv buffer [B*S, 3E] (q | k | v, head h at column h*Dh of each
// part), replacing the reference's per-(batch, head) SIMT kernels
// (src/kernel/cuda/mha.cu:18-122, :164-299) that materialise the full
// [B,H,S,S] probability tensor in HBM.  Scores never leave registers; the
// forward keeps the per-row log-sum-exp for the backward, which recomputes
// P.  The backward applies the 1/sqrt(Dh) factor to dQ and dK (the
// reference omits it, mha.cu:284-295).  Optional inverse RoPE on dq/dk at
// write-out (interleaved pairs, matching the forward rotation applied in
// the qkv GEMM epilogue).
//
// Tiles: 64 query rows x 64 keys per step, 4 warps x 16 rows, bf16
// mma.sync.m16n8k16 with fp32 accumulation; K/V (forward) and Q/dO
// (backward) tiles are double-buffered with cp.async; shared tiles are
// XOR-swizzled in 16-byte chunks so ldmatrix is conflict-free.
//
// fp32 path (reference API, mha.cuh:18-48): same semantics as the
// reference including the stored probabilities and the optional
// reference-exact backward without the scale factor.
#include <cfloat>
#include <cmath>
#include <cstdlib>

#include "common.cuh"

namespace zl {

namespace fa {

constexpr int TILE = 64;      // rows per tile (queries or keys)
constexpr int THREADS = 128;  // 4 warps
constexpr float LOG2E = 1.4426950408889634f;

// Shared memory of the kernels for head dim DH (bytes): rows of DH bf16.
template <int DH> __host__ __device__ constexpr int tile_bytes() { return TILE * DH * 2; }
template <int DH> __host__ __device__ constexpr int fwd_smem() { return 5 * tile_bytes<DH>(); }  // Q, K[2], V[2]
// K, V, Q[2], dO[2], dS^T [64][64], lse2[2][64], D[2][64]
template <int DH> __host__ __device__ constexpr int bwd_smem() { return 6 * tile_bytes<DH>() + TILE * 128 + 4 * TILE * 4; }

// Byte offset of element (row, col) in a swizzled tile with RW bf16 per row: 16-byte chunks are
// XOR-ed with (row & 7), so the 8 rows an ldmatrix phase reads hit 8 different bank groups.
template <int RW>
__device__ __forceinline__ uint32_t swz(int row, int col) {
  return (uint32_t)(row * (RW * 2) + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Loads a 64-row x DH-col bf16 tile whose row r starts at base + r*ld (elements) into swizzled smem.
// Rows >= valid_rows are zero-filled.
template <int DH>
__device__ __forceinline__ void load_tile(uint32_t smem, const __nv_bfloat16* base, int64_t ld, int valid_rows) {
  constexpr int CPR = DH / 8;  // 16-byte chunks per row
  for (int i = threadIdx.x; i < TILE * CPR; i += THREADS) {
    const int r = i / CPR, c = (i % CPR) * 8;
    const uint32_t dst = smem + swz<DH>(r, c);
    if (r < valid_rows) {
      cp_async16(dst, base + (int64_t)r * ld + c);
    } else {
      asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(dst), "r"(0));
    }
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (16 x 16) at rows [r0, r0+16), cols [c0, c0+16) of a row-major swizzled tile.
template <int RW>
__device__ __forceinline__ void load_a(uint32_t tile, int r0, int c0, uint32_t (&a)[4]) {
  const int l = threadIdx.x & 31;
  ldsm_x4(tile + swz<RW>(r0 + (l & 15), c0 + (l >> 4) * 8), a[0], a[1], a[2], a[3]);
}
// A fragment from a tile stored transposed: element (m, k) lives at [k][m].
template <int RW>
__device__ __forceinline__ void load_a_t(uint32_t tile, int m0, int k0, uint32_t (&a)[4]) {
  const int l = threadIdx.x & 31, i = l >> 3;
  const int k = k0 + (l & 7) + ((i >> 1) << 3), m = m0 + ((i & 1) << 3);
  ldsm_x4_t(tile + swz<RW>(k, m), a[0], a[1], a[2], a[3]);
}
// B fragments for two n-tiles [n0, n0+16) x k [k0, k0+16) from a tile stored [n][k].
template <int RW>
__device__ __forceinline__ void load_b_nk(uint32_t tile, int n0, int k0, uint32_t (&b)[4]) {
  const int l = threadIdx.x & 31;
  ldsm_x4(tile + swz<RW>(n0 + (l & 7) + ((l >> 4) << 3), k0 + ((l >> 3) & 1) * 8), b[0], b[1], b[2], b[3]);
}
// B fragments for two n-tiles from a tile stored [k][n] (transposed load).
template <int RW>
__device__ __forceinline__ void load_b_kn(uint32_t tile, int k0, int n0, uint32_t (&b)[4]) {
  const int l = threadIdx.x & 31;
  ldsm_x4_t(tile + swz<RW>(k0 + (l & 7) + (((l >> 3) & 1) << 3), n0 + ((l >> 4) << 3)), b[0], b[1], b[2], b[3]);
}

// ----------------------------------------------------------------- forward
template <int DH>
__global__ void __launch_bounds__(THREADS) fa_fwd_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                         __nv_bfloat16* __restrict__ out, float* __restrict__ lse,
                                                         int B, int S, int H, float scale_log2) {
  constexpr int TB = tile_bytes<DH>();
  constexpr int KD = DH / 16;  // k-steps over the head dim
  constexpr int ND = DH / 8;   // n-tiles of 8 over the head dim
  extern __shared__ __align__(128) uint8_t sm[];  // Q, K[2], V[2]
  const uint32_t sQ = smem_u32(sm), sK0 = sQ + TB, sV0 = sK0 + 2 * TB;
  const int E = H * DH;
  const int64_t ld = 3 * (int64_t)E;
  const int nq = (S + TILE - 1) / TILE;
  const int qb = nq - 1 - (int)(blockIdx.x % nq);  // heavy (late) blocks first
  const int bh = blockIdx.x / nq, b = bh / H, h = bh % H;
  const int q0 = qb * TILE;
  const __nv_bfloat16* base = qkv + (int64_t)b * S * ld;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  load_tile<DH>(sQ, base + (int64_t)q0 * ld + h * DH, ld, S - q0);
  load_tile<DH>(sK0, base + E + h * DH, ld, S);
  load_tile<DH>(sV0, base + 2 * E + h * DH, ld, S);
  cp_async_commit();

  float o[ND][4];
#pragma unroll
  for (int n = 0; n < ND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
  uint32_t qa[KD][4];

  const int nkv = qb + 1;
  for (int j = 0; j < nkv; ++j) {
    const int cur = j & 1;
    if (j + 1 < nkv) {
      const int k1 = (j + 1) * TILE;
      load_tile<DH>(sK0 + (cur ^ 1) * TB, base + (int64_t)k1 * ld + E + h * DH, ld, S - k1);
      load_tile<DH>(sV0 + (cur ^ 1) * TB, base + (int64_t)k1 * ld + 2 * E + h * DH, ld, S - k1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (j == 0) {
#pragma unroll
      for (int kk = 0; kk < KD; ++kk) load_a<DH>(sQ, warp * 16, kk * 16, qa[kk]);
    }
    const uint32_t sK = sK0 + cur * TB, sV = sV0 + cur * TB;
    // S = Q K^T  (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KD; ++kk)
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {
        uint32_t bf[4];
        load_b_nk<DH>(sK, n2 * 16, kk * 16, bf);
        mma16816(s[2 * n2], qa[kk], bf[0], bf[1]);
        mma16816(s[2 * n2 + 1], qa[kk], bf[2], bf[3]);
      }
    // scale (base 2), causal mask on the diagonal tile and for keys beyond S
    const int k0 = j * TILE;
    const int r_lo = q0 + warp * 16 + (lane >> 2), r_hi = r_lo + 8;
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + n * 8 + 2 * (lane & 3) + (e & 1);
        const int row = (e < 2) ? r_lo : r_hi;
        float v = s[n][e] * scale_log2;
        if (key > row || key >= S) v = -INFINITY;
        s[n][e] = v;
      }
    // online softmax
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float mx = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) mx = fmaxf(mx, fmaxf(s[n][2 * hr], s[n][2 * hr + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mnew = fmaxf(mrow[hr], mx);
      const float corr = (mnew == -INFINITY) ? 1.f : exp2f(mrow[hr] - mnew);
      float sum = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float p0 = (mnew == -INFINITY) ? 0.f : exp2f(s[n][2 * hr] - mnew);
        const float p1 = (mnew == -INFINITY) ? 0.f : exp2f(s[n][2 * hr + 1] - mnew);
        s[n][2 * hr] = p0;
        s[n][2 * hr + 1] = p1;
        sum += p0 + p1;
      }
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      lrow[hr] = lrow[hr] * corr + sum;
      mrow[hr] = mnew;
#pragma unroll
      for (int n = 0; n < ND; ++n) { o[n][2 * hr] *= corr; o[n][2 * hr + 1] *= corr; }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int n2 = 0; n2 < ND / 2; ++n2) {
        uint32_t bf[4];
        load_b_kn<DH>(sV, kk * 16, n2 * 16, bf);
        mma16816(o[2 * n2], pa, bf[0], bf[1]);
        mma16816(o[2 * n2 + 1], pa, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
  // write O / l and lse
  const int r_lo = q0 + warp * 16 + (lane >> 2);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = r_lo + hr * 8;
    if (row >= S) continue;
    const float inv = lrow[hr] > 0.f ? 1.f / lrow[hr] : 0.f;
    __nv_bfloat16* orow = out + ((int64_t)b * S + row) * E + h * DH;
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      const int c = n * 8 + 2 * (lane & 3);
      *reinterpret_cast<uint32_t*>(orow + c) = pack_bf16(o[n][2 * hr] * inv, o[n][2 * hr + 1] * inv);
    }
    if ((lane & 3) == 0)
      lse[((int64_t)b * H + h) * S + row] = (mrow[hr] + log2f(lrow[hr])) * 0.6931471805599453f;
  }
}

// ----------------------------------------------------------------- backward
// D[b,h,i] = sum_d dO[i,d] * O[i,d] and, when `nl` is given, nl[b,h,i] = -lse[b,h,i] * log2(e) (the
// exponent offset the tcgen05 kernel reads).  One thread per 8 consecutive elements of a token's
// row (16-byte loads of O and dO, at element offset 8 * thread index); the Dh/8 threads of a head
// reduce with shuffles.  Index arithmetic is 32-bit (the host checks B * S * H * Dh < 2^31).
// The same threads zero the fp32 dQ accumulator (T * E floats, 8 per thread) that the main pass then
// adds into, in place of a separate memset, and the first zeroes the main pass's unit counter.
__global__ void fa_bwd_pre_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ d_o,
                                  const float* __restrict__ lse, float* __restrict__ Dsum, float* __restrict__ nl,
                                  float* __restrict__ dq_zero, int* __restrict__ unit_ctr, int B, int S, int H,
                                  int DH) {
  const uint32_t cpt = (uint32_t)(H * DH) / 8u;  // chunks per token
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx == 0 && unit_ctr) *unit_ctr = 0;
  const bool live = idx < (uint32_t)B * (uint32_t)S * cpt;
  float s = 0.f;
  if (live) {
    const uint4 a = __ldg(reinterpret_cast<const uint4*>(o) + idx);
    const uint4 g = __ldg(reinterpret_cast<const uint4*>(d_o) + idx);
    float4* z = reinterpret_cast<float4*>(dq_zero) + (size_t)idx * 2;
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
    const uint32_t av[4] = {a.x, a.y, a.z, a.w}, gv[4] = {g.x, g.y, g.z, g.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 x = unpack_bf16(av[k]), y = unpack_bf16(gv[k]);
      s += x.x * y.x + x.y * y.y;
    }
  }
  // Dh/8 (8 or 16) consecutive lanes hold one head; E/8 is a multiple of 8, so groups never straddle warps
  for (int off = (DH / 8) >> 1; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const uint32_t per_head = (uint32_t)DH / 8u;
  if (live && (idx % per_head) == 0) {
    const uint32_t t = idx / cpt, c = idx - t * cpt;
    const uint32_t b = t / (uint32_t)S, i = t - b * (uint32_t)S;
    const uint32_t at = (b * (uint32_t)H + c / per_head) * (uint32_t)S + i;
    Dsum[at] = s;
    if (nl) nl[at] = -lse[at] * LOG2E;
  }
}

__device__ __forceinline__ void rope_inv_pair(float& x0, float& x1, const float* ct, const float* st, int pos,
                                              int pair, int half) {
  const float c = __ldg(ct + (int64_t)pos * half + pair), s = __ldg(st + (int64_t)pos * half + pair);
  const float a = x0, b = x1;
  x0 = a * c + b * s;
  x1 = -a * s + b * c;
}

// One CTA per (batch, head, 64-key block), four warps of 16 keys; dK / dV accumulate in registers
// over the query blocks, dQ goes through fp32 atomics.  At head dim 128 the K / V fragments are
// re-read from shared memory instead of kept in registers.
template <int DH>
__global__ void __launch_bounds__(THREADS) fa_bwd_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                         const __nv_bfloat16* __restrict__ d_o,
                                                         const float* __restrict__ lse,
                                                         const float* __restrict__ Dsum,
                                                         float* __restrict__ dq_acc,
                                                         __nv_bfloat16* __restrict__ d_qkv, const float* rope_cos,
                                                         const float* rope_sin, int B, int S, int H, float scale,
                                                         float scale_log2) {
  constexpr int TB = tile_bytes<DH>();
  constexpr int KD = DH / 16;
  constexpr int ND = DH / 8;
  constexpr bool CACHE_KV = (DH == 64);
  extern __shared__ __align__(128) uint8_t sm[];
  const uint32_t sK = smem_u32(sm), sV = sK + TB, sQ0 = sV + TB, sD0 = sQ0 + 2 * TB, sS = sD0 + 2 * TB;
  float* sL = reinterpret_cast<float*>(sm + 6 * TB + TILE * 128);  // [2][64] lse*log2e
  float* sDs = sL + 2 * TILE;                                        // [2][64] D
  const int E = H * DH;
  const int64_t ld = 3 * (int64_t)E;
  const int nk = (S + TILE - 1) / TILE;
  const int kb = (int)(blockIdx.x % nk);  // light (late key) blocks have fewer q blocks
  const int bh = blockIdx.x / nk, b = bh / H, h = bh % H;
  const int k0 = kb * TILE;
  const __nv_bfloat16* base = qkv + (int64_t)b * S * ld;
  const __nv_bfloat16* dob = d_o + (int64_t)b * S * E;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  auto load_q_block = [&](int qb, int buf) {
    const int q0 = qb * TILE;
    load_tile<DH>(sQ0 + buf * TB, base + (int64_t)q0 * ld + h * DH, ld, S - q0);
    load_tile<DH>(sD0 + buf * TB, dob + (int64_t)q0 * E + h * DH, E, S - q0);
    for (int i = threadIdx.x; i < TILE; i += THREADS) {
      const int q = q0 + i;
      sL[buf * TILE + i] = q < S ? lse[((int64_t)b * H + h) * S + q] * LOG2E : 0.f;
      sDs[buf * TILE + i] = q < S ? Dsum[((int64_t)b * H + h) * S + q] : 0.f;
    }
  };

  load_tile<DH>(sK, base + (int64_t)k0 * ld + E + h * DH, ld, S - k0);
  load_tile<DH>(sV, base + (int64_t)k0 * ld + 2 * E + h * DH, ld, S - k0);
  load_q_block(kb, 0);
  cp_async_commit();

  float dk[ND][4], dv[ND][4];
#pragma unroll
  for (int n = 0; n < ND; ++n)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[n][e] = dv[n][e] = 0.f;
  uint32_t ka[CACHE_KV ? KD : 1][4], va[CACHE_KV ? KD : 1][4];

  const int nq = nk;
  for (int qb = kb; qb < nq; ++qb) {
    const int cur = (qb - kb) & 1;
    if (qb + 1 < nq) {
      load_q_block(qb + 1, cur ^ 1);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (CACHE_KV && qb == kb) {
#pragma unroll
      for (int kk = 0; kk < KD; ++kk) {
        load_a<DH>(sK, warp * 16, kk * 16, ka[CACHE_KV ? kk : 0]);
        load_a<DH>(sV, warp * 16, kk * 16, va[CACHE_KV ? kk : 0]);
      }
    }
    const uint32_t sQ = sQ0 + cur * TB, sDO = sD0 + cur * TB;
    const float* Lq = sL + cur * TILE;
    const float* Dq = sDs + cur * TILE;
    const int q0 = qb * TILE;
    // S^T = K Q^T and dP^T = V dO^T  (16 keys x 64 queries per warp)
    float st[8][4], dpt[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[n][e] = dpt[n][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KD; ++kk) {
      uint32_t kf[4], vf[4];
      if constexpr (CACHE_KV) {
#pragma unroll
        for (int e = 0; e < 4; ++e) { kf[e] = ka[kk][e]; vf[e] = va[kk][e]; }
      } else {
        load_a<DH>(sK, warp * 16, kk * 16, kf);
        load_a<DH>(sV, warp * 16, kk * 16, vf);
      }
#pragma unroll
      for (int n2 = 0; n2 < 4; ++n2) {
        uint32_t bq[4], bd[4];
        load_b_nk<DH>(sQ, n2 * 16, kk * 16, bq);
        load_b_nk<DH>(sDO, n2 * 16, kk * 16, bd);
        mma16816(st[2 * n2], kf, bq[0], bq[1]);
        mma16816(st[2 * n2 + 1], kf, bq[2], bq[3]);
        mma16816(dpt[2 * n2], vf, bd[0], bd[1]);
        mma16816(dpt[2 * n2 + 1], vf, bd[2], bd[3]);
      }
    }
    // P^T and dS^T
    const int key_lo = k0 + warp * 16 + (lane >> 2);
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int ql = n * 8 + 2 * (lane & 3) + (e & 1);
        const int key = key_lo + ((e >> 1) << 3);
        const int q = q0 + ql;
        float p = exp2f(st[n][e] * scale_log2 - Lq[ql]);
        if (key > q || q >= S || key >= S) p = 0.f;
        st[n][e] = p;
        dpt[n][e] = p * (dpt[n][e] - Dq[ql]);
      }
    // dV += P^T dO ; dK += dS^T Q   (k = queries)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4], sa[4];
      pa[0] = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
      pa[1] = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
      pa[2] = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pa[3] = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      sa[0] = pack_bf16(dpt[2 * kk][0], dpt[2 * kk][1]);
      sa[1] = pack_bf16(dpt[2 * kk][2], dpt[2 * kk][3]);
      sa[2] = pack_bf16(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      sa[3] = pack_bf16(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int n2 = 0; n2 < ND / 2; ++n2) {
        uint32_t bd[4], bq[4];
        load_b_kn<DH>(sDO, kk * 16, n2 * 16, bd);
        load_b_kn<DH>(sQ, kk * 16, n2 * 16, bq);
        mma16816(dv[2 * n2], pa, bd[0], bd[1]);
        mma16816(dv[2 * n2 + 1], pa, bd[2], bd[3]);
        mma16816(dk[2 * n2], sa, bq[0], bq[1]);
        mma16816(dk[2 * n2 + 1], sa, bq[2], bq[3]);
      }
    }
    // dS^T -> shared [key][query] (bf16)
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int ql = n * 8 + 2 * (lane & 3);
      const int kl = warp * 16 + (lane >> 2);
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(sS + swz<64>(kl, ql)), "r"(pack_bf16(dpt[n][0], dpt[n][1])));
      asm volatile("st.shared.u32 [%0], %1;" ::"r"(sS + swz<64>(kl + 8, ql)), "r"(pack_bf16(dpt[n][2], dpt[n][3])));
    }
    __syncthreads();
    // dQ(64 q x DH) += dS (q x key) K (key x d): warp w owns queries [16w, 16w+16)
    float dq[ND][4];
#pragma unroll
    for (int n = 0; n < ND; ++n) dq[n][0] = dq[n][1] = dq[n][2] = dq[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t a[4];
      load_a_t<64>(sS, warp * 16, kk * 16, a);
#pragma unroll
      for (int n2 = 0; n2 < ND / 2; ++n2) {
        uint32_t bk[4];
        load_b_kn<DH>(sK, kk * 16, n2 * 16, bk);
        mma16816(dq[2 * n2], a, bk[0], bk[1]);
        mma16816(dq[2 * n2 + 1], a, bk[2], bk[3]);
      }
    }
    const int qr = q0 + warp * 16 + (lane >> 2);
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      const int q = qr + hr * 8;
      if (q >= S) continue;
      float* dst = dq_acc + ((int64_t)b * S + q) * E + h * DH;
#pragma unroll
      for (int n = 0; n < ND; ++n) {
        const int c = n * 8 + 2 * (lane & 3);
        atomicAdd(reinterpret_cast<float2*>(dst + c), make_float2(dq[n][2 * hr], dq[n][2 * hr + 1]));
      }
    }
    __syncthreads();
  }
  // write dK (scaled, optional inverse RoPE) and dV
  const int kr = k0 + warp * 16 + (lane >> 2);
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int key = kr + hr * 8;
    if (key >= S) continue;
    __nv_bfloat16* dkrow = d_qkv + ((int64_t)b * S + key) * ld + E + h * DH;
    __nv_bfloat16* dvrow = d_qkv + ((int64_t)b * S + key) * ld + 2 * E + h * DH;
#pragma unroll
    for (int n = 0; n < ND; ++n) {
      const int c = n * 8 + 2 * (lane & 3);
      float x0 = dk[n][2 * hr] * scale, x1 = dk[n][2 * hr + 1] * scale;
      if (rope_cos) rope_inv_pair(x0, x1, rope_cos, rope_sin, key, c >> 1, DH / 2);
      *reinterpret_cast<uint32_t*>(dkrow + c) = pack_bf16(x0, x1);
      *reinterpret_cast<uint32_t*>(dvrow + c) = pack_bf16(dv[n][2 * hr], dv[n][2 * hr + 1]);
    }
  }
}

// dQ = scale * dq_acc, rotated back by RoPE, into dq_out (`ld_out` elements per token: the Q columns
// of the packed gradient, or a separate [T, E] tensor).  dq_acc is [T, E]
// (token-major, the mma.sync kernel) or [B, H, S, Dh] (head-major, the tcgen05 kernel).  One thread
// per 8 consecutive elements (two 16-byte loads, one 16-byte store).
__global__ void fa_bwd_post_kernel(const float* __restrict__ dq_acc, __nv_bfloat16* __restrict__ dq_out, int ld_out,
                                   const float* rope_cos, const float* rope_sin, int64_t T, int S, int H,
                                   int DH, float scale, int head_major) {
  // 32-bit index arithmetic (the host checks T * E < 2^31): 64-bit divisions by runtime values
  // cost more issue slots than the thread's 48 bytes of traffic
  const uint32_t E = (uint32_t)(H * DH);
  const uint32_t idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint32_t)T * (E / 8u)) return;
  const uint32_t t = idx / (E / 8u);
  const uint32_t c = (idx - t * (E / 8u)) * 8u;
  const uint32_t bb = t / (uint32_t)S, pos = t - bb * (uint32_t)S;
  const uint32_t hh = c / (uint32_t)DH, cd = c - hh * (uint32_t)DH;
  const uint32_t src = head_major ? ((bb * (uint32_t)H + hh) * (uint32_t)S + pos) * (uint32_t)DH + cd : idx * 8u;
  const float4 v0 = __ldg(reinterpret_cast<const float4*>(dq_acc + src));
  const float4 v1 = __ldg(reinterpret_cast<const float4*>(dq_acc + src) + 1);
  float x[8] = {v0.x * scale, v0.y * scale, v0.z * scale, v0.w * scale,
                v1.x * scale, v1.y * scale, v1.z * scale, v1.w * scale};
  if (rope_cos) {
    // the chunk's four rotation pairs are consecutive in the [S, Dh/2] tables: one float4 of each
    const uint32_t r = pos * (uint32_t)(DH / 2) + (cd >> 1);
    const float4 cv = __ldg(reinterpret_cast<const float4*>(rope_cos + r));
    const float4 sv = __ldg(reinterpret_cast<const float4*>(rope_sin + r));
    const float cs[4] = {cv.x, cv.y, cv.z, cv.w}, sn[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float a = x[2 * k], b = x[2 * k + 1];
      x[2 * k] = a * cs[k] + b * sn[k];
      x[2 * k + 1] = -a * sn[k] + b * cs[k];
    }
  }
  uint4 u;
  u.x = pack_bf16(x[0], x[1]); u.y = pack_bf16(x[2], x[3]); u.z = pack_bf16(x[4], x[5]); u.w = pack_bf16(x[6], x[7]);
  *reinterpret_cast<uint4*>(dq_out + (size_t)t * (uint32_t)ld_out + c) = u;
}

}  // namespace fa

// ============================================================== fp32 reference API
// One warp per query row (b, h, i).  Pass 1: row max.  Pass 2: exp and sum
// (unnormalised probabilities go to `scores` when given).  Pass 3: O = P V.
// Finally `scores` is normalised in place, as mha.cu:102-106 leaves it.
__global__ void mha_fwd_f32_kernel(const float* __restrict__ Q, const float* __restrict__ K,
                                   const float* __restrict__ V, float* __restrict__ out, float* __restrict__ scores,
                                   const uint8_t* __restrict__ mask, int B, int S, int H, int Dh, int causal,
                                   float scale) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= (int64_t)B * H * S) return;  // warp-uniform
  const int lane = threadIdx.x & 31;
  const int i = (int)(row % S);
  const int h = (int)((row / S) % H);
  const int b = (int)(row / ((int64_t)S * H));
  const int E = H * Dh;
  const float* q = Q + ((int64_t)b * S + i) * E + h * Dh;
  float* sc = scores ? scores + (((int64_t)b * H + h) * S + i) * S : nullptr;
  auto keep = [&](int j) { return !(causal && j > i) && !(mask && !mask[(int64_t)i * S + j]); };
  auto dot = [&](int j) {  // warp-collective
    const float* k = K + ((int64_t)b * S + j) * E + h * Dh;
    float d = 0.f;
    for (int x = lane; x < Dh; x += 32) d = fmaf(q[x], k[x], d);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    return d * scale;
  };
  float mx = -FLT_MAX;
  for (int j = 0; j < S; ++j)
    if (keep(j)) mx = fmaxf(mx, dot(j));
  float sum = 0.f;
  for (int j = 0; j < S; ++j) {
    float e = 0.f;
    if (keep(j)) { e = expf(dot(j) - mx); sum += e; }
    if (sc && lane == 0) sc[j] = e;
  }
  if (sum == 0.f) sum = 1e-20f;  // mha.cu:103
  const float inv = 1.f / sum;
  __syncwarp();
  for (int x0 = 0; x0 < Dh; x0 += 32) {
    const int x = x0 + lane;
    float o = 0.f;
    for (int j = 0; j < S; ++j) {
      if (!keep(j)) continue;
      const float e = sc ? sc[j] : expf(dot(j) - mx);
      if (x < Dh) o = fmaf(e * inv, V[((int64_t)b * S + j) * E + h * Dh + x], o);
    }
    if (x < Dh) out[((int64_t)b * S + i) * E + h * Dh + x] = o;
  }
  __syncwarp();
  if (sc)
    for (int j = lane; j < S; j += 32) sc[j] = sc[j] * inv;
}

// Backward from stored probabilities P (mha.cu:164-299).
// dV[j] = sum_i P[i,j] dO[i]: one warp per key row.
__global__ void mha_bwd_dv_f32_kernel(const float* __restrict__ dO, const float* __restrict__ P,
                                      const uint8_t* __restrict__ mask, float* __restrict__ dV, int B, int S, int H,
                                      int Dh, int causal) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= (int64_t)B * H * S) return;
  const int lane = threadIdx.x & 31;
  const int j = (int)(row % S), h = (int)((row / S) % H), b = (int)(row / ((int64_t)S * H));
  const int E = H * Dh;
  const float* Pb = P + ((int64_t)b * H + h) * S * S;
  for (int x = lane; x < Dh; x += 32) {
    float acc = 0.f;
    for (int i = 0; i < S; ++i) {
      if (causal && j > i) continue;
      if (mask && !mask[(int64_t)i * S + j]) continue;
      const float p = Pb[(int64_t)i * S + j];
      if (p == 0.f) continue;
      acc = fmaf(p, dO[((int64_t)b * S + i) * E + h * Dh + x], acc);
    }
    dV[((int64_t)b * S + j) * E + h * Dh + x] = acc;
  }
}
// dS row i, dQ[i] accumulated in registers, dK[j] via atomics (dK pre-zeroed): one warp per query row.
__global__ void mha_bwd_dqk_f32_kernel(const float* __restrict__ dO, const float* __restrict__ Q,
                                       const float* __restrict__ K, const float* __restrict__ V,
                                       const float* __restrict__ P, const uint8_t* __restrict__ mask,
                                       float* __restrict__ dQ, float* __restrict__ dK, int B, int S, int H, int Dh,
                                       int causal, float ds_scale) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (row >= (int64_t)B * H * S) return;
  const int lane = threadIdx.x & 31;
  const int i = (int)(row % S), h = (int)((row / S) % H), b = (int)(row / ((int64_t)S * H));
  const int E = H * Dh;
  const float* Pb = P + ((int64_t)b * H + h) * S * S + (int64_t)i * S;
  const float* go = dO + ((int64_t)b * S + i) * E + h * Dh;
  auto g_of = [&](int j) {  // warp-collective dO_i . V_j
    const float* v = V + ((int64_t)b * S + j) * E + h * Dh;
    float d = 0.f;
    for (int x = lane; x < Dh; x += 32) d = fmaf(go[x], v[x], d);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) d += __shfl_xor_sync(0xffffffffu, d, off);
    return d;
  };
  auto keep = [&](int j) { return !(causal && j > i) && !(mask && !mask[(int64_t)i * S + j]); };
  float spg = 0.f;
  for (int j = 0; j < S; ++j) {
    if (!keep(j)) continue;
    const float p = Pb[j];
    if (p == 0.f) continue;
    spg += p * g_of(j);
  }
  float dq[4] = {0.f, 0.f, 0.f, 0.f};  // Dh <= 128
  const float* qi = Q + ((int64_t)b * S + i) * E + h * Dh;
  for (int j = 0; j < S; ++j) {
    if (!keep(j)) continue;
    const float p = Pb[j];
    if (p == 0.f) continue;
    const float ds = p * (g_of(j) - spg) * ds_scale;
    const float* kj = K + ((int64_t)b * S + j) * E + h * Dh;
    float* dkj = dK + ((int64_t)b * S + j) * E + h * Dh;
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int x = lane + 32 * t;
      if (x < Dh) {
        dq[t] = fmaf(ds, kj[x], dq[t]);
        atomicAdd(dkj + x, ds * qi[x]);
      }
    }
  }
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const int x = lane + 32 * t;
    if (x < Dh) dQ[((int64_t)b * S + i) * E + h * Dh + x] = dq[t];
  }
}

}  // namespace zl

// ============================================================== C ABI
namespace zl {
bool fa_fwd_tc_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int B, int S, int H, int Dh,
                      cudaStream_t st, zl_status* status);
bool fa_bwd_tc_supported(const void* qkv, const void* d_o, const void* dq_acc, const void* d_qkv, int S, int Dh);
zl_status fa_bwd_tc_launch(const __nv_bfloat16* qkv, const __nv_bfloat16* d_o, const float* nl, const float* Dsum,
                           float* dq_acc, __nv_bfloat16* d_qkv, const float* rope_cos, const float* rope_sin,
                           int* unit_ctr, int B, int S, int H, int Dh, cudaStream_t st);
bool fa_fwd_tc_launch3(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, int ld,
                       __nv_bfloat16* out, float* lse, int B, int S, int H, int Dh, cudaStream_t st, zl_status* status);
bool fa_bwd_tc_supported3(const void* q, const void* k, const void* v, int ld_in, const void* d_o, const void* dq_acc,
                          const void* dk, const void* dv, int ld_out, int S, int Dh);
zl_status fa_bwd_tc_launch3(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, int ld_in,
                            const __nv_bfloat16* d_o, const float* nl, const float* Dsum, float* dq_acc,
                            __nv_bfloat16* dk, __nv_bfloat16* dv, int ld_out, const float* rope_cos,
                            const float* rope_sin, int* unit_ctr, int B, int S, int H, int Dh, float dk_scale,
                            cudaStream_t st);
}
using namespace zl;

namespace {
// ZL_ATTENTION_KERNEL=mma forces the mma.sync kernels (kept for shapes the tcgen05 kernels do not
// cover); read on every call so that one process can run both.
bool force_mma_sync() {
  const char* e = getenv("ZL_ATTENTION_KERNEL");
  return e && e[0] == 'm';
}
}  // namespace

extern "C" zl_status zl_attention_forward_bf16(const zl_bf16* qkv, zl_bf16* o, float* lse, int batch, int seq_len,
                                               int num_heads, int head_dim, zl_stream stream) {
  if (batch <= 0 || seq_len <= 0 || num_heads <= 0) return set_error(ZL_EINVAL, "attention: invalid sizes");
  if (head_dim != 64 && head_dim != 128)
    return set_error(ZL_EUNSUPPORTED, "attention: head_dim %d (supported: 64, 128)", head_dim);
  if (!qkv || !o || !lse) return set_error(ZL_EINVAL, "attention: null pointer");
  if (!force_mma_sync()) {
    zl_status st = ZL_OK;
    if (fa_fwd_tc_launch(reinterpret_cast<const __nv_bfloat16*>(qkv), reinterpret_cast<__nv_bfloat16*>(o), lse, batch,
                         seq_len, num_heads, head_dim, (cudaStream_t)stream, &st))
      return st;
  }
  const int nq = (seq_len + fa::TILE - 1) / fa::TILE;
  const float scale_log2 = (1.0f / sqrtf((float)head_dim)) * fa::LOG2E;
  const unsigned grid = (unsigned)((int64_t)batch * num_heads * nq);
  auto launch = [&](auto kern, int smem) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kern<<<grid, fa::THREADS, smem, (cudaStream_t)stream>>>(reinterpret_cast<const __nv_bfloat16*>(qkv),
                                                            reinterpret_cast<__nv_bfloat16*>(o), lse, batch, seq_len,
                                                            num_heads, scale_log2);
  };
  if (head_dim == 64) launch(fa::fa_fwd_kernel<64>, fa::fwd_smem<64>());
  else launch(fa::fa_fwd_kernel<128>, fa::fwd_smem<128>());
  return check_launch("fa_fwd_kernel");
}

// dq accumulator [B*S, H*Dh], D and nl [B, H, S], then 16 bytes holding the backward's unit counter
extern "C" int64_t zl_attention_workspace_floats(int batch, int seq_len, int num_heads, int head_dim) {
  return (int64_t)batch * seq_len * num_heads * head_dim + 2 * (int64_t)batch * num_heads * seq_len + 4;
}

namespace zl {
// The backward of zl_attention_backward_bf16; ev0 / ev1 (may be null) are recorded just before and
// after its main kernel, as graph event nodes when the stream is being captured.
zl_status attention_backward_bf16(const zl_bf16* qkv, const zl_bf16* o, const zl_bf16* d_o, const float* lse,
                                  zl_bf16* d_qkv, float* workspace, int batch, int seq_len, int num_heads,
                                  int head_dim, const float* rope_cos, const float* rope_sin, zl_stream stream,
                                  cudaEvent_t ev0, cudaEvent_t ev1);
}  // namespace zl

extern "C" zl_status zl_attention_backward_bf16(const zl_bf16* qkv, const zl_bf16* o, const zl_bf16* d_o,
                                                const float* lse, zl_bf16* d_qkv, float* workspace, int batch,
                                                int seq_len, int num_heads, int head_dim, const float* rope_cos,
                                                const float* rope_sin, zl_stream stream) {
  return zl::attention_backward_bf16(qkv, o, d_o, lse, d_qkv, workspace, batch, seq_len, num_heads, head_dim, rope_cos,
                                     rope_sin, stream, nullptr, nullptr);
}

zl_status zl::attention_backward_bf16(const zl_bf16* qkv, const zl_bf16* o, const zl_bf16* d_o, const float* lse,
                                      zl_bf16* d_qkv, float* workspace, int batch, int seq_len, int num_heads,
                                      int head_dim, const float* rope_cos, const float* rope_sin, zl_stream stream,
                                      cudaEvent_t ev0, cudaEvent_t ev1) {
  if (batch <= 0 || seq_len <= 0 || num_heads <= 0) return set_error(ZL_EINVAL, "attention: invalid sizes");
  if (head_dim != 64 && head_dim != 128)
    return set_error(ZL_EUNSUPPORTED, "attention: head_dim %d (supported: 64, 128)", head_dim);
  if (!qkv || !o || !d_o || !lse || !d_qkv || !workspace) return set_error(ZL_EINVAL, "attention bwd: null pointer");
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return set_error(ZL_EINVAL, "attention bwd: rope tables");
  // the backward kernels read the rotation tables four pairs at a time (16-byte loads)
  if (((reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 15) != 0)
    return set_error(ZL_EINVAL, "attention bwd: rope tables must be 16-byte aligned");
  // the D pass reads o and d_o, and zeroes the workspace's dQ accumulator, 16 bytes at a time
  if (((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(d_o) | reinterpret_cast<uintptr_t>(workspace)) &
       15) != 0)
    return set_error(ZL_EINVAL, "attention bwd: o, d_o and workspace must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t T = (int64_t)batch * seq_len;
  const int E = num_heads * head_dim;
  if (T * E >= ((int64_t)1 << 31)) return set_error(ZL_EUNSUPPORTED, "attention bwd: batch*seq*embed must be < 2^31");
  float* dq_acc = workspace;
  float* Dsum = workspace + T * E;
  float* nl = Dsum + (int64_t)batch * num_heads * seq_len;
  int* unit_ctr = reinterpret_cast<int*>(nl + (int64_t)batch * num_heads * seq_len);
  const bool tc = !force_mma_sync() && fa_bwd_tc_supported(qkv, d_o, dq_acc, d_qkv, seq_len, head_dim);
  // the dq accumulator starts at zero (both backward kernels add into it): the pre pass zeroes it
  const int64_t chunks = T * (E / 8);
  fa::fa_bwd_pre_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(o), reinterpret_cast<const __nv_bfloat16*>(d_o), lse, Dsum,
      tc ? nl : nullptr, dq_acc, unit_ctr, batch, seq_len, num_heads, head_dim);
  zl_status s = check_launch("fa_bwd_pre_kernel");
  if (s != ZL_OK) return s;
  const float scale = 1.0f / sqrtf((float)head_dim);
  if (ev0) record_timing_event(ev0, st);
  if (tc) {
    s = fa_bwd_tc_launch(reinterpret_cast<const __nv_bfloat16*>(qkv), reinterpret_cast<const __nv_bfloat16*>(d_o), nl,
                         Dsum, dq_acc, reinterpret_cast<__nv_bfloat16*>(d_qkv), rope_cos, rope_sin, unit_ctr, batch,
                         seq_len, num_heads, head_dim, st);
    if (s != ZL_OK) return s;
  } else {
    const int nk = (seq_len + fa::TILE - 1) / fa::TILE;
    const unsigned grid = (unsigned)((int64_t)batch * num_heads * nk);
    auto launch = [&](auto kern, int smem) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      kern<<<grid, fa::THREADS, smem, st>>>(reinterpret_cast<const __nv_bfloat16*>(qkv),
                                            reinterpret_cast<const __nv_bfloat16*>(d_o), lse, Dsum, dq_acc,
                                            reinterpret_cast<__nv_bfloat16*>(d_qkv), rope_cos, rope_sin, batch,
                                            seq_len, num_heads, scale, scale * fa::LOG2E);
    };
    if (head_dim == 64) launch(fa::fa_bwd_kernel<64>, fa::bwd_smem<64>());
    else launch(fa::fa_bwd_kernel<128>, fa::bwd_smem<128>());
    s = check_launch("fa_bwd_kernel");
    if (s != ZL_OK) return s;
  }
  if (ev1) record_timing_event(ev1, st);
  fa::fa_bwd_post_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(
      dq_acc, reinterpret_cast<__nv_bfloat16*>(d_qkv), 3 * E, rope_cos, rope_sin, T, seq_len, num_heads, head_dim,
      scale, tc ? 1 : 0);
  return check_launch("fa_bwd_post_kernel");
}

// ------------------------------------------------------------ reference-style bf16 attention (mha.cuh:18-48)
// State kept between the forward and the backward, laid out in the caller's `state` buffer (the
// reference API's attention_scores, B*H*S*S elements): the per-row log-sum-exp, a copy of the output
// (the backward's D = rowsum(dO * O) needs it and the reference backward is not given O), then the
// backward's fp32 dQ accumulator and row vectors.  Each region starts on a 256-byte boundary.
namespace {
struct MhaState {
  size_t lse, o, dq, dsum, nl, ctr, fwd_end, total;
};
MhaState mha_state_layout(int64_t B, int64_t S, int64_t H, int64_t Dh) {
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  const size_t rows = (size_t)B * H * S, te = (size_t)B * S * H * Dh;
  MhaState m;
  m.lse = 0;
  m.o = up(m.lse + rows * 4);
  m.fwd_end = up(m.o + te * 2);
  m.dq = m.fwd_end;
  m.dsum = up(m.dq + te * 4);
  m.nl = up(m.dsum + rows * 4);
  m.ctr = up(m.nl + rows * 4);  // the backward's unit counter
  m.total = up(m.ctr + 16);
  return m;
}
zl_status mha_bf16_check(const void* q, const void* k, const void* v, const void* state, int64_t B, int64_t S,
                         int64_t H, int64_t Dh, int causal, const uint8_t* mask, size_t state_bytes, bool bwd) {
  if (B <= 0 || S <= 0 || H <= 0 || Dh <= 0) return set_error(ZL_EINVAL, "mha bf16: invalid sizes");
  if (!q || !k || !v || !state) return set_error(ZL_EINVAL, "mha bf16: null pointer");
  if (!causal || mask)
    return set_error(ZL_EUNSUPPORTED, "mha bf16: the flash-attention path is causal and takes no mask");
  if ((Dh != 64 && Dh != 128) || S % 128 != 0)
    return set_error(ZL_EUNSUPPORTED, "mha bf16: head_dim %lld (64 or 128) and seq_len %lld (a multiple of 128)",
                     (long long)Dh, (long long)S);
  if (B * S * H * Dh >= ((int64_t)1 << 31)) return set_error(ZL_EUNSUPPORTED, "mha bf16: batch*seq*embed >= 2^31");
  const MhaState m = mha_state_layout(B, S, H, Dh);
  const size_t need = bwd ? m.total : m.fwd_end;
  if (state_bytes < need)
    return set_error(ZL_EINVAL, "mha bf16: the state buffer holds %zu bytes, %zu needed", state_bytes, need);
  if (reinterpret_cast<uintptr_t>(state) & 255) return set_error(ZL_EINVAL, "mha bf16: state must be 256-byte aligned");
  return ZL_OK;
}
}  // namespace

extern "C" size_t zl_mha_state_bytes_bf16(int64_t batch, int64_t seq_len, int64_t num_heads, int64_t head_dim) {
  return mha_state_layout(batch, seq_len, num_heads, head_dim).total;
}

extern "C" zl_status zl_mha_forward_bf16(const zl_bf16* Q, const zl_bf16* K, const zl_bf16* V, zl_bf16* attn_output,
                                         void* state, size_t state_bytes, const uint8_t* mask, int64_t batch,
                                         int64_t seq_len, int64_t num_heads, int64_t head_dim, int is_causal,
                                         zl_stream stream) {
  zl_status st = mha_bf16_check(Q, K, V, state, batch, seq_len, num_heads, head_dim, is_causal, mask, state_bytes,
                                false);
  if (st != ZL_OK) return st;
  if (!attn_output) return set_error(ZL_EINVAL, "mha bf16: null output");
  const MhaState m = mha_state_layout(batch, seq_len, num_heads, head_dim);
  uint8_t* base = static_cast<uint8_t*>(state);
  const int E = (int)(num_heads * head_dim);
  cudaStream_t cs = (cudaStream_t)stream;
  zl_status ks = ZL_OK;
  if (!fa_fwd_tc_launch3(reinterpret_cast<const __nv_bfloat16*>(Q), reinterpret_cast<const __nv_bfloat16*>(K),
                         reinterpret_cast<const __nv_bfloat16*>(V), E, reinterpret_cast<__nv_bfloat16*>(attn_output),
                         reinterpret_cast<float*>(base + m.lse), (int)batch, (int)seq_len, (int)num_heads,
                         (int)head_dim, cs, &ks))
    return set_error(ZL_EUNSUPPORTED, "mha bf16: Q, K, V must be 16-byte aligned");
  if (ks != ZL_OK) return ks;
  const cudaError_t e = cudaMemcpyAsync(base + m.o, attn_output, (size_t)batch * seq_len * E * 2,
                                        cudaMemcpyDeviceToDevice, cs);
  return e == cudaSuccess ? ZL_OK : set_error(ZL_ECUDA, "mha bf16: output copy: %s", cudaGetErrorString(e));
}

extern "C" zl_status zl_mha_backward_bf16(const zl_bf16* d_attn_output, const zl_bf16* Q, const zl_bf16* K,
                                          const zl_bf16* V, void* state, size_t state_bytes, const uint8_t* mask,
                                          zl_bf16* d_Q, zl_bf16* d_K, zl_bf16* d_V, int64_t batch, int64_t seq_len,
                                          int64_t num_heads, int64_t head_dim, int is_causal, int reference_semantics,
                                          zl_stream stream) {
  zl_status st = mha_bf16_check(Q, K, V, state, batch, seq_len, num_heads, head_dim, is_causal, mask, state_bytes,
                                true);
  if (st != ZL_OK) return st;
  if (!d_attn_output || !d_Q || !d_K || !d_V) return set_error(ZL_EINVAL, "mha bf16: null gradient pointer");
  const MhaState m = mha_state_layout(batch, seq_len, num_heads, head_dim);
  uint8_t* base = static_cast<uint8_t*>(state);
  float* lse = reinterpret_cast<float*>(base + m.lse);
  const __nv_bfloat16* o = reinterpret_cast<const __nv_bfloat16*>(base + m.o);
  float* dq_acc = reinterpret_cast<float*>(base + m.dq);
  float* Dsum = reinterpret_cast<float*>(base + m.dsum);
  float* nl = reinterpret_cast<float*>(base + m.nl);
  int* unit_ctr = reinterpret_cast<int*>(base + m.ctr);
  const int B = (int)batch, S = (int)seq_len, H = (int)num_heads, Dh = (int)head_dim, E = H * Dh;
  if (!fa_bwd_tc_supported3(Q, K, V, E, d_attn_output, dq_acc, d_K, d_V, E, S, Dh) ||
      (reinterpret_cast<uintptr_t>(d_Q) & 15))
    return set_error(ZL_EUNSUPPORTED, "mha bf16: tensors must be 16-byte aligned");
  cudaStream_t cs = (cudaStream_t)stream;
  const int64_t T = (int64_t)B * S, chunks = T * (E / 8);
  fa::fa_bwd_pre_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, cs>>>(
      o, reinterpret_cast<const __nv_bfloat16*>(d_attn_output), lse, Dsum, nl, dq_acc, unit_ctr, B, S, H, Dh);
  st = check_launch("fa_bwd_pre_kernel");
  if (st != ZL_OK) return st;
  // the reference backward leaves out the softmax scale in dQ and dK (mha.cu:284-295)
  const float g_scale = reference_semantics ? 1.0f : 1.0f / sqrtf((float)Dh);
  st = fa_bwd_tc_launch3(reinterpret_cast<const __nv_bfloat16*>(Q), reinterpret_cast<const __nv_bfloat16*>(K),
                         reinterpret_cast<const __nv_bfloat16*>(V), E,
                         reinterpret_cast<const __nv_bfloat16*>(d_attn_output), nl, Dsum, dq_acc,
                         reinterpret_cast<__nv_bfloat16*>(d_K), reinterpret_cast<__nv_bfloat16*>(d_V), E, nullptr,
                         nullptr, unit_ctr, B, S, H, Dh, g_scale, cs);
  if (st != ZL_OK) return st;
  fa::fa_bwd_post_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, cs>>>(
      dq_acc, reinterpret_cast<__nv_bfloat16*>(d_Q), E, nullptr, nullptr, T, S, H, Dh, g_scale, 1);
  return check_launch("fa_bwd_post_kernel");
}

extern "C" zl_status zl_mha_forward_f32(const float* Q, const float* K, const float* V, float* attn_output,
                                        float* attention_scores, const uint8_t* mask, int64_t batch, int64_t seq_len,
                                        int64_t num_heads, int64_t head_dim, int is_causal, zl_stream stream) {
  if (batch <= 0 || seq_len <= 0 || num_heads <= 0 || head_dim <= 0)
    return set_error(ZL_EINVAL, "mha_forward: invalid sizes");  // mha.cu:133-135
  if (head_dim > 128) return set_error(ZL_EUNSUPPORTED, "mha_forward: head_dim > 128");
  const int64_t rows = batch * num_heads * seq_len;
  mha_fwd_f32_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, (cudaStream_t)stream>>>(
      Q, K, V, attn_output, attention_scores, mask, (int)batch, (int)seq_len, (int)num_heads, (int)head_dim,
      is_causal, 1.0f / sqrtf((float)head_dim));
  return check_launch("mha_fwd_f32_kernel");
}

extern "C" zl_status zl_mha_backward_f32(const float* d_attn_output, const float* Q, const float* K, const float* V,
                                         const float* attention_scores, const uint8_t* mask, float* d_Q, float* d_K,
                                         float* d_V, int64_t batch, int64_t seq_len, int64_t num_heads,
                                         int64_t head_dim, int is_causal, int reference_semantics,
                                         zl_stream stream) {
  if (batch <= 0 || seq_len <= 0 || num_heads <= 0 || head_dim <= 0)
    return set_error(ZL_EINVAL, "cuda_mha_backward: invalid sizes");  // mha.cu:312-314
  if (head_dim > 128) return set_error(ZL_EUNSUPPORTED, "mha_backward: head_dim > 128");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t rows = batch * num_heads * seq_len;
  const size_t bytes = (size_t)batch * seq_len * num_heads * head_dim * sizeof(float);
  if (cudaMemsetAsync(d_K, 0, bytes, st) != cudaSuccess) return check_launch("mha_backward memset");
  mha_bwd_dv_f32_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(d_attn_output, attention_scores, mask, d_V,
                                                                      (int)batch, (int)seq_len, (int)num_heads,
                                                                      (int)head_dim, is_causal);
  zl_status s = check_launch("mha_bwd_dv_f32_kernel");
  if (s != ZL_OK) return s;
  const float ds_scale = reference_semantics ? 1.0f : 1.0f / sqrtf((float)head_dim);
  mha_bwd_dqk_f32_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(d_attn_output, Q, K, V, attention_scores, mask,
                                                                       d_Q, d_K, (int)batch, (int)seq_len,
                                                                       (int)num_heads, (int)head_dim, is_causal,
                                                                       ds_scale);
  return check_launch("mha_bwd_dqk_f32_kernel");
}

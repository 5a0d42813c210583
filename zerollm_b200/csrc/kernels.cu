// kernels.cu -- memory-bound kernels: norms, embedding, cross-entropy,
// optimizers, element-wise ops and reductions.
//
// Design: 128-bit vectorised global access (8 bf16 / 4 fp32 per load), one
// warp per row for row-wise ops on d_model-wide rows, shared-memory staging
// for vocabulary-wide rows, and two-stage (partials -> reduce) column and
// scalar reductions so results are independent of scheduling.
// The fp32 reference-API kernels keep the reference's per-element
// semantics (file:line cited on each).
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <mutex>
#include <type_traits>

#include "common.cuh"

namespace zl {
int sm_count_current();  // gemm.cu

// ------------------------------------------------------------------ errors
static thread_local char g_err[512] = "";

zl_status set_error(zl_status code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}
zl_status check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(ZL_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return ZL_OK;
}

constexpr int kMaxRowChunks = 8;  // rows up to 8 * 256 = 2048 elements held in registers by one warp

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ void load8(const __nv_bfloat16* p, float (&v)[8]) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y), c = unpack_bf16(u.z), d = unpack_bf16(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y), c = unpack_bf16(u.z), d = unpack_bf16(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}
__device__ __forceinline__ void store8(__nv_bfloat16* p, const float (&v)[8]) {
  uint4 u;
  u.x = pack_bf16(v[0], v[1]); u.y = pack_bf16(v[2], v[3]); u.z = pack_bf16(v[4], v[5]); u.w = pack_bf16(v[6], v[7]);
  *reinterpret_cast<uint4*>(p) = u;
}
__device__ __forceinline__ void load8f(const float* p, float (&v)[8]) {
  float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// ================================================================== norms (bf16 rows)
// kind 0: LayerNorm (layernorm.cu:6-76 semantics: biased variance), kind 1: RMSNorm.
// One warp per row; the warps stay resident (grid-stride over rows) and fetch the next row's
// packed input while the current one is reduced and written, so each SM keeps a row per warp in
// flight.
template <int KIND, int kMaxChunks>
__global__ void __launch_bounds__(256) norm_fwd_bf16_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const float* __restrict__ g, const float* __restrict__ b,
                                                          __nv_bfloat16* __restrict__ y, float* __restrict__ mean_out,
                                                          float* __restrict__ rstd_out, int64_t M, int N, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t nwarps = (int64_t)gridDim.x * (blockDim.x >> 5);
  int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  uint4 nxt[kMaxChunks];
  auto fetch = [&](int64_t r) {
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < N) nxt[c] = __ldg(reinterpret_cast<const uint4*>(x + r * N + col));
    }
  };
  if (row < M) fetch(row);
  for (; row < M; row += nwarps) {
    float v[kMaxChunks][8];
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c)
      if ((c * 32 + lane) * 8 < N) unpack8(nxt[c], v[c]);
    if (row + nwarps < M) fetch(row + nwarps);
    float s = 0.f;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c)
      if ((c * 32 + lane) * 8 < N)
#pragma unroll
        for (int j = 0; j < 8; ++j) s += KIND == 0 ? v[c][j] : v[c][j] * v[c][j];
    s = warp_sum(s);
    float mu = 0.f, rs;
    if (KIND == 0) {
      mu = s / (float)N;
      float q = 0.f;
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c)
        if ((c * 32 + lane) * 8 < N)
#pragma unroll
          for (int j = 0; j < 8; ++j) { const float d = v[c][j] - mu; q += d * d; }
      q = warp_sum(q);
      rs = rsqrtf(q / (float)N + eps);
    } else {
      rs = rsqrtf(s / (float)N + eps);
    }
    if (lane == 0) {
      if (mean_out) mean_out[row] = mu;
      if (rstd_out) rstd_out[row] = rs;
    }
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < N) {
        float gv[8], o[8];
        load8f(g + col, gv);
        if (KIND == 0) {
          float bv[8];
          load8f(b + col, bv);
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = (v[c][j] - mu) * rs * gv[j] + bv[j];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) o[j] = v[c][j] * rs * gv[j];
        }
        store8(y + row * N + col, o);
      }
    }
  }
}

// Backward: one warp per row (resident warps, next row prefetched).  Per-block column partials go
// to `part` [gridDim.x][NP] with NP = N * (1 + LayerNorm + COL): dgamma | dbeta (LayerNorm) |
// column sums of dx (COL: the bias gradient of the layer whose output this norm consumed).
// Rows of up to 512 columns combine their eight warps' partials in shared memory; wider rows use
// shared-memory atomics.
// STAGES > 0: each warp streams its rows through a ring of STAGES shared-memory slots filled by
// 1-D bulk copies (x row and dy row per slot), so that STAGES rows per warp are in flight instead of
// the one prefetched row of the register path (STAGES == 0).  Dynamic shared memory: the rings
// [8][STAGES][2][N] bf16, their barriers [8][STAGES], then the partial accumulators.
template <int KIND, int kMaxChunks, bool COL, int STAGES>
__global__ void __launch_bounds__(256) norm_bwd_bf16_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ dy,
                                                          const float* __restrict__ g, const float* __restrict__ mean,
                                                          const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                                                          float* __restrict__ part, int64_t M, int N,
                                                          float* __restrict__ sum0, float* __restrict__ sum1,
                                                          float* __restrict__ sum2) {
  constexpr int NK = 1 + (KIND == 0 ? 1 : 0) + (COL ? 1 : 0);  // partial sets
  extern __shared__ __align__(16) uint8_t nb_smem[];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5, warps = blockDim.x >> 5;
  const size_t ring_bytes = STAGES > 0 ? (size_t)8 * STAGES * 4 * N : 0;
  uint8_t* ring = nb_smem + (size_t)w * STAGES * 4 * N;
  uint64_t* bars = reinterpret_cast<uint64_t*>(nb_smem + ring_bytes) + w * (STAGES > 0 ? STAGES : 1);
  float* sacc = reinterpret_cast<float*>(nb_smem + ring_bytes + (STAGES > 0 ? 8 * STAGES * 8 : 0));  // [8][NK*N] or [NK*N]
  const bool tree = N <= 512;
  const int NP = NK * N;
  if (!tree) {
    for (int i = threadIdx.x; i < NP; i += blockDim.x) sacc[i] = 0.f;
    __syncthreads();
  }
  float pg[kMaxChunks][8], pb[kMaxChunks][8], pc[kMaxChunks][8];
#pragma unroll
  for (int c = 0; c < kMaxChunks; ++c)
#pragma unroll
    for (int j = 0; j < 8; ++j) pg[c][j] = pb[c][j] = pc[c][j] = 0.f;
  const int64_t nwarps = (int64_t)gridDim.x * warps;
  int64_t row = (int64_t)blockIdx.x * warps + w;
  // register path: rows of up to 512 columns prefetch the next row; wider rows would run out of registers
  constexpr bool PREFETCH = STAGES == 0 && kMaxChunks <= 2;
  // rows of up to 512 columns keep gamma in registers for the whole launch and x-hat, dy * gamma of
  // the row between the two passes (reloading gamma twice per row cost more L1 traffic than the
  // row itself); wider rows reload and recompute them
  constexpr bool KEEP = kMaxChunks <= 2;
  float gl[KEEP ? kMaxChunks : 1][8];
  // KEEP rows run their per-element arithmetic on column pairs (paired fp32 instructions, each lane
  // rounding like the scalar one): gamma, the dgamma / dbeta / column-sum accumulators and the
  // row's x-hat, dy * gamma are held as pairs
  uint64_t gl2[KEEP ? kMaxChunks : 1][4], pg2[KEEP ? kMaxChunks : 1][4], pb2[KEEP ? kMaxChunks : 1][4],
      pc2[KEEP ? kMaxChunks : 1][4];
  if constexpr (KEEP) {
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < N) load8f(g + col, gl[c]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        gl2[c][i] = f2_pack(gl[c][2 * i], gl[c][2 * i + 1]);
        pg2[c][i] = pb2[c][i] = pc2[c][i] = 0ull;  // +0.0f in both halves
      }
    }
  }
  uint4 nx[kMaxChunks], nd[kMaxChunks];
  auto fetch = [&](int64_t r) {
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < N) {
        nx[c] = __ldg(reinterpret_cast<const uint4*>(x + r * N + col));
        nd[c] = __ldg(reinterpret_cast<const uint4*>(dy + r * N + col));
      }
    }
  };
  // staged path: row k of this warp (row + k * nwarps) goes to slot k % STAGES
  auto issue = [&](int64_t k) {
    const int64_t r = row + k * nwarps;
    if (r >= M) return;
    const int sl = (int)(k % STAGES);
    uint8_t* dst = ring + (size_t)sl * 4 * N;
    mbar_arrive_expect_tx(&bars[sl], (uint32_t)(4 * N));
    bulk_copy_g2s(dst, x + r * N, (uint32_t)(2 * N), &bars[sl]);
    bulk_copy_g2s(dst + 2 * N, dy + r * N, (uint32_t)(2 * N), &bars[sl]);
  };
  if constexpr (STAGES > 0) {
    if (lane == 0) {
      for (int i = 0; i < STAGES; ++i) mbar_init(&bars[i], 1);
      fence_mbar_init();
      for (int i = 0; i < STAGES; ++i) issue(i);
    }
    __syncwarp();
  }
  if (PREFETCH && row < M) fetch(row);
  // the row statistics of this warp's next 32 rows, one per lane (a load per row would put a memory
  // round trip in front of every row's arithmetic)
  float mu_l = 0.f, rs_l = 0.f;
  auto stats = [&](int64_t k0) {
    const int64_t rr = row + (k0 + lane) * nwarps;
    if (rr < M) {
      rs_l = rstd[rr];
      if (KIND == 0) mu_l = mean[rr];
    }
  };
  stats(0);
  int64_t k = 0;
  for (; row + k * nwarps < M; ++k) {
    const int64_t r = row + k * nwarps;
    if (k > 0 && (k & 31) == 0) stats(k);
    const float mu = KIND == 0 ? __shfl_sync(0xffffffffu, mu_l, (int)(k & 31)) : 0.f;
    const float rs = __shfl_sync(0xffffffffu, rs_l, (int)(k & 31));
    // keep only the packed row; both passes unpack it again (registers, not arithmetic, limit
    // the resident warps here)
    uint4 cx[kMaxChunks], cd[kMaxChunks];
    if constexpr (STAGES > 0) {
      const int sl = (int)(k % STAGES);
      if (!bounded_wait_warp(&bars[sl], (uint32_t)((k / STAGES) & 1), DEV_TIMEOUT_FULL)) break;
      const uint8_t* src = ring + (size_t)sl * 4 * N;
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < N) {
          cx[c] = *reinterpret_cast<const uint4*>(src + col * 2);
          cd[c] = *reinterpret_cast<const uint4*>(src + 2 * N + col * 2);
        }
      }
      __syncwarp();
      if (lane == 0) issue(k + STAGES);  // the slot has been read by every lane
    } else {
      if (!PREFETCH) fetch(r);
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) { cx[c] = nx[c]; cd[c] = nd[c]; }
      if (PREFETCH && r + nwarps < M) fetch(r + nwarps);
    }
    float s1 = 0.f, s2 = 0.f;
    uint64_t xhk2[KEEP ? kMaxChunks : 1][4], ak2[KEEP ? kMaxChunks : 1][4];
    if constexpr (KEEP) {
      const uint64_t mu2 = f2_pack(mu, mu), rs2 = f2_pack(rs, rs);
      uint64_t s12 = 0ull, s22 = 0ull;
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < N) {
          const uint32_t xw[4] = {cx[c].x, cx[c].y, cx[c].z, cx[c].w}, dw[4] = {cd[c].x, cd[c].y, cd[c].z, cd[c].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            // bf16 pair -> fp32 pair (element 2i in the low half of the word)
            const uint64_t x2 = f2_pack(__uint_as_float(xw[i] << 16), __uint_as_float(xw[i] & 0xffff0000u));
            const uint64_t d2 = f2_pack(__uint_as_float(dw[i] << 16), __uint_as_float(dw[i] & 0xffff0000u));
            const uint64_t xh2 = KIND == 0 ? mul2(sub2(x2, mu2), rs2) : mul2(x2, rs2);
            const uint64_t a2 = mul2(d2, gl2[c][i]);
            s12 = add2(s12, a2);
            s22 = fma2(a2, xh2, s22);
            pg2[c][i] = fma2(d2, xh2, pg2[c][i]);
            if (KIND == 0) pb2[c][i] = add2(pb2[c][i], d2);
            xhk2[c][i] = xh2;
            ak2[c][i] = a2;
          }
        }
      }
      float e, o;
      f2_unpack(s12, e, o);
      s1 = e + o;
      f2_unpack(s22, e, o);
      s2 = e + o;
    } else {
#pragma unroll
      for (int c = 0; c < kMaxChunks; ++c) {
        const int col = (c * 32 + lane) * 8;
        if (col < N) {
          float gv[8], xv[8], dv[8];
          load8f(g + col, gv);
          unpack8(cx[c], xv);
          unpack8(cd[c], dv);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xh = (xv[j] - mu) * rs;
            const float a = dv[j] * gv[j];
            s1 += a;
            s2 += a * xh;
            pg[c][j] += dv[j] * xh;
            if (KIND == 0) pb[c][j] += dv[j];
          }
        }
      }
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    const float invN = 1.f / (float)N;
    // dx = rs * (dy*g - s1/N - x-hat * s2/N)  (LayerNorm; RMSNorm has no s1 term)
    const float c1 = KIND == 0 ? rs * s1 * invN : 0.f, c2 = rs * s2 * invN;
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < N) {
        float o[8];
        if constexpr (KEEP) {
          const uint64_t rs2 = f2_pack(rs, rs), nc1 = f2_pack(-c1, -c1), nc2 = f2_pack(-c2, -c2);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint64_t o2 = fma2(xhk2[c][i], nc2, fma2(rs2, ak2[c][i], nc1));
            if (COL) pc2[c][i] = add2(pc2[c][i], o2);
            f2_unpack(o2, o[2 * i], o[2 * i + 1]);
          }
        } else {
          float gv[8], xv[8], dv[8];
          load8f(g + col, gv);
          unpack8(cx[c], xv);
          unpack8(cd[c], dv);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float xh = (xv[j] - mu) * rs;
            o[j] = fmaf(-xh, c2, fmaf(rs, dv[j] * gv[j], -c1));
          }
        }
        if constexpr (!KEEP) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if (COL) pc[c][j] += o[j];
        }
        store8(dx + r * N + col, o);
      }
    }
  }
  if constexpr (STAGES > 0) {  // after a timeout: no copy may still be landing when the block exits
    if (lane == 0)
      for (int64_t j = k; j < k + STAGES; ++j)
        if (row + j * nwarps < M) bounded_wait(&bars[j % STAGES], (uint32_t)((j / STAGES) & 1), DEV_TIMEOUT_FULL);
    __syncwarp();
  }
  if constexpr (KEEP) {
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        f2_unpack(pg2[c][i], pg[c][2 * i], pg[c][2 * i + 1]);
        f2_unpack(pb2[c][i], pb[c][2 * i], pb[c][2 * i + 1]);
        f2_unpack(pc2[c][i], pc[c][2 * i], pc[c][2 * i + 1]);
      }
  }
  // block partials: [dgamma | dbeta | column sums]
  auto put = [&](float* base, bool atomic) {
#pragma unroll
    for (int c = 0; c < kMaxChunks; ++c) {
      const int col = (c * 32 + lane) * 8;
      if (col < N)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          int k = 0;
          if (atomic) atomicAdd(&base[col + j], pg[c][j]); else base[col + j] = pg[c][j];
          if (KIND == 0) { ++k; if (atomic) atomicAdd(&base[k * N + col + j], pb[c][j]); else base[k * N + col + j] = pb[c][j]; }
          if (COL) { ++k; if (atomic) atomicAdd(&base[k * N + col + j], pc[c][j]); else base[k * N + col + j] = pc[c][j]; }
        }
    }
  };
  // The block's sums go to `part` (row blockIdx.x, reduced by a second launch in a fixed order), or,
  // when sum0 is given, are added straight into sum0 | sum1 | sum2 (columns [0,N) | [N,2N) | [2N,3N)
  // of the partial set) with 16-byte atomics: no second launch, additions in any order.
  auto emit4 = [&](int i, float4 t) {
    if (sum0) {
      float* o = i < N ? sum0 + i : (i < 2 * N ? sum1 + (i - N) : sum2 + (i - 2 * N));
      atomicAdd(reinterpret_cast<float4*>(o), t);
    } else {
      *reinterpret_cast<float4*>(part + (int64_t)blockIdx.x * NP + i) = t;
    }
  };
  if (tree) {
    put(sacc + w * NP, false);
    __syncthreads();
    for (int i = threadIdx.x * 4; i < NP; i += blockDim.x * 4) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = 0; k < warps; ++k) {
        const float4 v = *reinterpret_cast<const float4*>(sacc + k * NP + i);
        t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
      }
      emit4(i, t);
    }
  } else {
    put(sacc, true);
    __syncthreads();
    for (int i = threadIdx.x * 4; i < NP; i += blockDim.x * 4) emit4(i, *reinterpret_cast<const float4*>(sacc + i));
  }
}

// Sums per-block partials [nb][stride] into out0 (columns [0, N)) and, when out1 is given, out1
// (columns [N, 2N)), accumulating.  One block per 32 columns: its 32 warps take every 32nd
// partial row (four loads in flight), then warp 0 adds the 32 warp sums in a fixed order, so the
// result does not depend on timing.
constexpr int kReduceWarps = 32;
__global__ void __launch_bounds__(kReduceWarps * 32) reduce_partials_kernel(const float* __restrict__ part, int nb, int N,
                                                                         int stride, float* __restrict__ out0,
                                                                         float* __restrict__ out1,
                                                                         float* __restrict__ out2) {
  __shared__ float red[kReduceWarps][33];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int ncols = (out2 ? 3 : out1 ? 2 : 1) * N;
  const int c = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (c < ncols) {
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int k = w;
    for (; k + 3 * kReduceWarps < nb; k += 4 * kReduceWarps) {
      a0 += part[(int64_t)k * stride + c];
      a1 += part[(int64_t)(k + kReduceWarps) * stride + c];
      a2 += part[(int64_t)(k + 2 * kReduceWarps) * stride + c];
      a3 += part[(int64_t)(k + 3 * kReduceWarps) * stride + c];
    }
    for (; k < nb; k += kReduceWarps) a0 += part[(int64_t)k * stride + c];
    s = (a0 + a1) + (a2 + a3);
  }
  red[w][lane] = s;
  __syncthreads();
  if (w == 0 && c < ncols) {
    float t = 0.f;
#pragma unroll 8
    for (int j = 0; j < kReduceWarps; ++j) t += red[j][lane];
    if (c < N) out0[c] += t;
    else if (c < 2 * N) out1[c - N] += t;
    else out2[c - 2 * N] += t;
  }
}
// Partial columns [0, N) -> out0, [N, 2N) -> out1, [2N, 3N) -> out2 (out1 / out2 may be null, in
// which case the later ones are too).
void launch_reduce_partials(const float* part, int nb, int N, int stride, float* out0, float* out1, cudaStream_t st,
                            float* out2 = nullptr) {
  const int ncols = (out2 ? 3 : out1 ? 2 : 1) * N;
  reduce_partials_kernel<<<(ncols + 31) / 32, kReduceWarps * 32, 0, st>>>(part, nb, N, stride, out0, out1, out2);
}

int norm_bwd_blocks(int64_t M) {
  int64_t nb = (M + 31) / 32;  // >= 32 rows per block (8 warps x 4 rows)
  return (int)(nb < 592 ? nb : 592);
}

// ================================================================== embedding
// Model form: x[t] = bf16(E[id] + P[t % S]); invalid id -> zero row.
__global__ void embed_fwd_bf16_kernel(const int32_t* __restrict__ ids, const float* __restrict__ table,
                                      const float* __restrict__ pos, __nv_bfloat16* __restrict__ out, int64_t T, int S,
                                      int D, int V) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  const int id = ids[t];
  const bool valid = id >= 0 && id < V;
  const int s = (int)(t % S);
  for (int col = lane * 8; col < D; col += 256) {
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (valid) {
      load8f(table + (int64_t)id * D + col, v);
      if (pos) {
        float p[8];
        load8f(pos + (int64_t)s * D + col, p);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] += p[j];
      }
    }
    store8(out + t * D + col, v);
  }
}
__global__ void embed_bwd_bf16_kernel(const int32_t* __restrict__ ids, const __nv_bfloat16* __restrict__ dx,
                                      float* __restrict__ dtable, int64_t T, int D, int V) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int lane = threadIdx.x & 31;
  const int id = ids[t];
  if (id < 0 || id >= V) return;
  for (int col = lane * 8; col < D; col += 256) {
    float v[8];
    load8(dx + t * D + col, v);
    float4* dst = reinterpret_cast<float4*>(dtable + (int64_t)id * D + col);
    atomicAdd(dst, make_float4(v[0], v[1], v[2], v[3]));
    atomicAdd(dst + 1, make_float4(v[4], v[5], v[6], v[7]));
  }
}
// Reference form (embedding.cu:6-30): out[idx] = table[id*D+k] + pos[s*D+k]; skip s >= max_seq_len or invalid id.
__global__ void embed_fwd_f32_kernel(const int32_t* __restrict__ ids, const float* __restrict__ table,
                                     const float* __restrict__ pos, float* __restrict__ out, int B, int S, int D, int V,
                                     int max_seq_len) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * S * D) return;
  const int k = (int)(idx % D);
  const int64_t t = idx / D;
  const int s = (int)(t % S);
  if (s >= max_seq_len) return;
  const int id = ids[t];
  if (id < 0 || id >= V) return;
  out[idx] = table[(int64_t)id * D + k] + pos[(int64_t)s * D + k];
}
// embedding.cu:33-53
__global__ void embed_bwd_f32_kernel(const int32_t* __restrict__ ids, const float* __restrict__ dout,
                                     float* __restrict__ dtable, int B, int S, int D, int V) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * S * D) return;
  const int k = (int)(idx % D);
  const int id = ids[idx / D];
  if (id < 0 || id >= V) return;
  atomicAdd(&dtable[(int64_t)id * D + k], dout[idx]);
}

// ================================================================== cross-entropy
// One CTA per row; the row is staged in shared memory (fp32).
__global__ void ce_fused_bf16_kernel(__nv_bfloat16* __restrict__ logits, const int32_t* __restrict__ targets, int V,
                                     float cap, float grad_scale, float* __restrict__ loss_rows) {
  extern __shared__ float srow[];
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  __nv_bfloat16* x = logits + r * V;
  const int tid = threadIdx.x, nt = blockDim.x;
  float mx = -INFINITY;
  const int nv = V / 8;
  for (int i = tid; i < nv; i += nt) {
    float v[8];
    load8(x + i * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) { srow[i * 8 + j] = v[j]; mx = fmaxf(mx, v[j]); }
  }
  for (int i = nv * 8 + tid; i < V; i += nt) { const float v = __bfloat162float(x[i]); srow[i] = v; mx = fmaxf(mx, v); }
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  if (tid < 32) {
    float m = tid < (nt >> 5) ? red[tid] : -INFINITY;
    m = warp_max(m);
    if (tid == 0) red[0] = m;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float s = 0.f;
  for (int i = tid; i < V; i += nt) s += __expf(srow[i] - mx);
  s = warp_sum(s);
  if ((tid & 31) == 0) red[tid >> 5] = s;
  __syncthreads();
  if (tid < 32) {
    float v = tid < (nt >> 5) ? red[tid] : 0.f;
    v = warp_sum(v);
    if (tid == 0) red[0] = v;
  }
  __syncthreads();
  const float lse = mx + logf(red[0]);
  const int t = targets[r];
  const bool valid = t >= 0 && t < V;
  if (tid == 0) loss_rows[r] = valid ? fminf(lse - srow[t], cap) : 0.f;
  for (int i = tid; i < nv; i += nt) {
    float o[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = i * 8 + j;
      o[j] = (__expf(srow[c] - lse) - (c == t ? 1.f : 0.f)) * grad_scale;
    }
    store8(x + i * 8, o);
  }
  for (int i = nv * 8 + tid; i < V; i += nt)
    x[i] = __float2bfloat16_rn((__expf(srow[i] - lse) - (i == t ? 1.f : 0.f)) * grad_scale);
}

// The same loss and gradient with the row held in registers (vocab <= 8 * 256 * MAXV): one exponential
// per logit, reused for the row sum and the gradient, and no shared-memory copy of the row.  Every
// thread keeps up to MAXV vectors of 8 logits (vector i of the row goes to thread i % 256).
template <int MAXV>
__global__ void __launch_bounds__(256) ce_fused_reg_bf16_kernel(__nv_bfloat16* __restrict__ logits,
                                                               const int32_t* __restrict__ targets, int V, float cap,
                                                               float grad_scale, float* __restrict__ loss_rows) {
  __shared__ float red[8];
  const int64_t r = blockIdx.x;
  __nv_bfloat16* x = logits + r * V;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int nv = V / 8;
  const int t = targets[r];
  const bool valid = t >= 0 && t < V;
  // the target logit, read before any thread overwrites the row with its gradient
  const float xt = (tid == 0 && valid) ? __bfloat162float(x[t]) : 0.f;
  float e[MAXV][8];
  float mx = -INFINITY;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = tid + k * 256;
    if (i < nv) {
      load8(x + i * 8, e[k]);
#pragma unroll
      for (int j = 0; j < 8; ++j) mx = fmaxf(mx, e[k][j]);
    }
  }
  mx = warp_max(mx);
  if (lane == 0) red[w] = mx;
  __syncthreads();
  mx = red[0];
#pragma unroll
  for (int k = 1; k < 8; ++k) mx = fmaxf(mx, red[k]);
  __syncthreads();
  float sum = 0.f;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = tid + k * 256;
    if (i < nv) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        e[k][j] = __expf(e[k][j] - mx);
        sum += e[k][j];
      }
    }
  }
  sum = warp_sum(sum);
  if (lane == 0) red[w] = sum;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += red[k];  // fixed order
  const float lse = mx + logf(tot);
  if (tid == 0) loss_rows[r] = valid ? fminf(lse - xt, cap) : 0.f;
  const float inv = 1.f / tot;
#pragma unroll
  for (int k = 0; k < MAXV; ++k) {
    const int i = tid + k * 256;
    if (i < nv) {
      float o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (e[k][j] * inv - (i * 8 + j == t ? 1.f : 0.f)) * grad_scale;
      store8(x + i * 8, o);
    }
  }
}

// Deterministic mean of `n` values (single CTA, fixed order tree).
__global__ void mean_kernel(const float* __restrict__ v, int64_t n, float* __restrict__ out, float denom) {
  __shared__ double red[1024];
  double s = 0.0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += v[i];
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = (float)(red[0] / denom);
}

// The reference API's kernels are written once for fp32 and bf16 storage; arithmetic is fp32, and
// the fp32 instances are plain loads and stores (the bf16 ones round each stored value to nearest).
__device__ __forceinline__ float ldv(const float* p) { return *p; }
__device__ __forceinline__ float ldv(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void stv(float* p, float v) { *p = v; }
__device__ __forceinline__ void stv(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void atomic_addv(float* p, float v) { atomicAdd(p, v); }
__device__ __forceinline__ void atomic_addv(__nv_bfloat16* p, float v) { atomicAdd(p, __float2bfloat16_rn(v)); }

// softmax.cu:12-65 (one CTA per row).  fp32 rows keep the reference's order (exponentials stored,
// then divided); bf16 rows recompute the exponential in the last pass instead of storing it rounded.
template <typename T = float>
__global__ void softmax_f32_kernel(const T* __restrict__ in, T* __restrict__ out, int N) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  const T* x = in + r * N;
  T* y = out + r * N;
  const int tid = threadIdx.x, nt = blockDim.x;
  float mx = -FLT_MAX;
  for (int i = tid; i < N; i += nt) mx = fmaxf(mx, ldv(x + i));
  mx = warp_max(mx);
  if ((tid & 31) == 0) red[tid >> 5] = mx;
  __syncthreads();
  if (tid < 32) {
    float m = tid < (nt >> 5) ? red[tid] : -FLT_MAX;
    m = warp_max(m);
    if (tid == 0) red[0] = m;
  }
  __syncthreads();
  mx = red[0];
  __syncthreads();
  float s = 0.f;
  for (int i = tid; i < N; i += nt) {
    const float e = expf(ldv(x + i) - mx);
    if constexpr (std::is_same<T, float>::value) y[i] = e;
    s += e;
  }
  s = warp_sum(s);
  if ((tid & 31) == 0) red[tid >> 5] = s;
  __syncthreads();
  if (tid < 32) {
    float v = tid < (nt >> 5) ? red[tid] : 0.f;
    v = warp_sum(v);
    if (tid == 0) red[0] = v;
  }
  __syncthreads();
  const float sum = red[0];
  if constexpr (std::is_same<T, float>::value) {
    for (int i = tid; i < N; i += nt) y[i] = y[i] / sum;
  } else {
    for (int i = tid; i < N; i += nt) stv(y + i, expf(ldv(x + i) - mx) / sum);
  }
}
// cross_entropy.cu:5-31
__global__ void ce_bwd_f32_kernel(float* __restrict__ d, const float* __restrict__ p, const int32_t* __restrict__ t,
                                  int rows, int C) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)rows * C) return;
  const int r = (int)(idx / C), c = (int)(idx % C);
  const int tg = t[r];
  float v = p[idx];
  if (tg >= 0 && tg < C && c == tg) v = p[idx] - 1.0f;
  d[idx] = v / (float)rows;
}
// cross_entropy.cpp:59-76 (host loop moved to the device): one CTA, fixed-order
// reduction of -log(max(p[r, t_r], eps)) over all rows, divided by rows.
__global__ void ce_loss_f32_kernel(const float* __restrict__ p, const int32_t* __restrict__ t, int rows, int C,
                                   float eps, float* __restrict__ out) {
  __shared__ double red[1024];
  double s = 0.0;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const int tg = t[r];
    if (tg >= 0 && tg < C) s += -logf(fmaxf(p[(int64_t)r * C + tg], eps));
  }
  red[threadIdx.x] = s;
  __syncthreads();
  for (int o = blockDim.x / 2; o > 0; o >>= 1) {
    if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = (float)(red[0] / rows);
}

// ================================================================== optimizers
// adamw.cu:26-73 per element, gradient scaled by grad_scale, optional bf16 shadow.
__global__ void adamw_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                             float* __restrict__ v, __nv_bfloat16* __restrict__ pb, int64_t n, float lr, float wd,
                             float b1, float b2, float eps, float bc1, float bc2, float gs) {
  const int64_t i4 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i4 >= n) return;
  const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
  if (i4 + 4 <= n && ((reinterpret_cast<uintptr_t>(p + i4) | reinterpret_cast<uintptr_t>(g + i4)) & 15) == 0) {
    float4 P = *reinterpret_cast<float4*>(p + i4), G = *reinterpret_cast<const float4*>(g + i4);
    float4 Mv = *reinterpret_cast<float4*>(m + i4), Vv = *reinterpret_cast<float4*>(v + i4);
    float pa[4] = {P.x, P.y, P.z, P.w}, ga[4] = {G.x, G.y, G.z, G.w}, ma[4] = {Mv.x, Mv.y, Mv.z, Mv.w},
          va[4] = {Vv.x, Vv.y, Vv.z, Vv.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float gv = ga[j] * gs;
      ma[j] = b1 * ma[j] + omb1 * gv;
      va[j] = b2 * va[j] + omb2 * gv * gv;
      const float step = lr * (ma[j] / bc1) / (sqrtf(va[j] / bc2) + eps);
      const float decay = wd != 0.f ? lr * wd * pa[j] : 0.f;
      pa[j] = pa[j] - (decay + step);
    }
    *reinterpret_cast<float4*>(p + i4) = make_float4(pa[0], pa[1], pa[2], pa[3]);
    *reinterpret_cast<float4*>(m + i4) = make_float4(ma[0], ma[1], ma[2], ma[3]);
    *reinterpret_cast<float4*>(v + i4) = make_float4(va[0], va[1], va[2], va[3]);
    if (pb) {
      uint2 u;
      u.x = pack_bf16(pa[0], pa[1]);
      u.y = pack_bf16(pa[2], pa[3]);
      *reinterpret_cast<uint2*>(pb + i4) = u;
    }
  } else {
    for (int64_t i = i4; i < n && i < i4 + 4; ++i) {
      const float gv = g[i] * gs;
      const float mv = b1 * m[i] + omb1 * gv;
      const float vv = b2 * v[i] + omb2 * gv * gv;
      m[i] = mv;
      v[i] = vv;
      const float step = lr * (mv / bc1) / (sqrtf(vv / bc2) + eps);
      const float decay = wd != 0.f ? lr * wd * p[i] : 0.f;
      p[i] = p[i] - (decay + step);
      if (pb) pb[i] = __float2bfloat16_rn(p[i]);
    }
  }
}
// adam.cu:13-57
__global__ void adam_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                            float* __restrict__ v, int64_t n, float lr, float b1, float b2, float eps, float bc1,
                            float bc2) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = g[i];
  const float mv = b1 * m[i] + (1.0f - b1) * gv;
  const float vv = b2 * v[i] + (1.0f - b2) * gv * gv;
  m[i] = mv;
  v[i] = vv;
  p[i] -= lr * (mv / bc1) / (sqrtf(vv / bc2) + eps);
}
// sgd.cu:14-57
__global__ void sgd_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ vel, int64_t n,
                           float lr, float momentum, float wd) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float pv = p[i];
  float gv = g[i];
  if (wd != 0.f) gv += wd * pv;
  if (momentum != 0.f && vel) {
    const float vv = momentum * vel[i] + gv;
    vel[i] = vv;
    gv = vv;
  }
  p[i] = pv - lr * gv;
}

// ================================================================== element-wise (reference API)

template <typename T>
__global__ void add_kernel(const T* __restrict__ a, const T* __restrict__ b, T* __restrict__ o, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) stv(o + i, ldv(a + i) + ldv(b + i));
}
template <typename T>
__global__ void add_inplace_kernel(T* __restrict__ a, const T* __restrict__ b, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) stv(a + i, ldv(a + i) + ldv(b + i));
}
template <typename T>
__global__ void relu_fwd_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    const float v = ldv(x + i);
    stv(y + i, v > 0 ? v : 0.f);
  }
}
template <typename T>
__global__ void relu_bwd_kernel(const T* __restrict__ x, const T* __restrict__ gy, T* __restrict__ gx, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) stv(gx + i, ldv(x + i) > 0 ? ldv(gy + i) : 0.f);
}
// adamw.cu:26-73 on bf16 parameters and moments: fp32 arithmetic, each stored value rounded.
__global__ void adamw_bf16_kernel(__nv_bfloat16* __restrict__ p, const __nv_bfloat16* __restrict__ g,
                                  __nv_bfloat16* __restrict__ m, __nv_bfloat16* __restrict__ v, int64_t n, float lr,
                                  float wd, float b1, float b2, float eps, float bc1, float bc2) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float gv = ldv(g + i), pv = ldv(p + i);
  const float mv = b1 * ldv(m + i) + (1.0f - b1) * gv;
  const float vv = b2 * ldv(v + i) + (1.0f - b2) * gv * gv;
  const float step = lr * (mv / bc1) / (sqrtf(vv / bc2) + eps);
  const float decay = wd != 0.f ? lr * wd * pv : 0.f;
  stv(p + i, pv - (decay + step));
  stv(m + i, mv);
  stv(v + i, vv);
}
// 32x32 tiles through shared memory: coalesced reads and writes.
__global__ void transpose_kernel(const float* __restrict__ in, float* __restrict__ out, int rows, int cols) {
  __shared__ float t[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int r = r0 + k, c = c0 + threadIdx.x;
    if (r < rows && c < cols) t[k][threadIdx.x] = in[(int64_t)r * cols + c];
  }
  __syncthreads();
  for (int k = threadIdx.y; k < 32; k += blockDim.y) {
    const int c = c0 + k, r = r0 + threadIdx.x;
    if (r < rows && c < cols) out[(int64_t)c * rows + r] = t[threadIdx.x][k];
  }
}
__global__ void f32_to_bf16_kernel(const float* __restrict__ x, __nv_bfloat16* __restrict__ y, int64_t n) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(x[i]);
}

// LayerNorm / RMSNorm on fp32 rows (reference API): one warp per row, dgamma/dbeta
// accumulated per block in shared memory and added with one atomic per column per block.
template <int KIND, typename T = float>
__global__ void norm_fwd_f32_kernel(const T* __restrict__ x, const T* __restrict__ g, const T* __restrict__ b,
                                    T* __restrict__ y, T* __restrict__ mean, T* __restrict__ rstd, int64_t M,
                                    int N, float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= M) return;
  const int lane = threadIdx.x & 31;
  const T* xr = x + row * N;
  float s = 0.f;
  for (int i = lane; i < N; i += 32) s += KIND == 0 ? ldv(xr + i) : ldv(xr + i) * ldv(xr + i);
  s = warp_sum(s);
  float mu = 0.f, rs;
  if (KIND == 0) {
    mu = s / (float)N;
    float q = 0.f;
    for (int i = lane; i < N; i += 32) { const float d = ldv(xr + i) - mu; q += d * d; }
    q = warp_sum(q);
    rs = rsqrtf(q / (float)N + eps);
  } else {
    rs = rsqrtf(s / (float)N + eps);
  }
  if (lane == 0) {
    if (mean) stv(mean + row, mu);
    if (rstd) stv(rstd + row, rs);
  }
  for (int i = lane; i < N; i += 32)
    stv(y + row * N + i, KIND == 0 ? (ldv(xr + i) - mu) * rs * ldv(g + i) + ldv(b + i) : ldv(xr + i) * rs * ldv(g + i));
}
template <int KIND, typename T = float>
__global__ void norm_bwd_f32_kernel(const T* __restrict__ x, const T* __restrict__ dy, const T* __restrict__ g,
                                    const T* __restrict__ mean, const T* __restrict__ rstd,
                                    T* __restrict__ dx, T* __restrict__ dg, T* __restrict__ db, int64_t M,
                                    int N) {
  extern __shared__ float sacc[];  // [2N]
  for (int i = threadIdx.x; i < 2 * N; i += blockDim.x) sacc[i] = 0.f;
  __syncthreads();
  const int lane = threadIdx.x & 31, warps = blockDim.x >> 5;
  for (int64_t row = (int64_t)blockIdx.x * warps + (threadIdx.x >> 5); row < M; row += (int64_t)gridDim.x * warps) {
    const float mu = KIND == 0 ? ldv(mean + row) : 0.f, rs = ldv(rstd + row);
    const T* xr = x + row * N;
    const T* dr = dy + row * N;
    float s1 = 0.f, s2 = 0.f;
    for (int i = lane; i < N; i += 32) {
      const float xh = (ldv(xr + i) - mu) * rs, a = ldv(dr + i) * ldv(g + i);
      s1 += a;
      s2 += a * xh;
      atomicAdd(&sacc[i], ldv(dr + i) * xh);
      if (KIND == 0) atomicAdd(&sacc[N + i], ldv(dr + i));
    }
    s1 = warp_sum(s1);
    s2 = warp_sum(s2);
    const float invN = 1.f / (float)N;
    for (int i = lane; i < N; i += 32) {
      const float xh = (ldv(xr + i) - mu) * rs, a = ldv(dr + i) * ldv(g + i);
      stv(dx + row * N + i, KIND == 0 ? rs * (a - s1 * invN - xh * s2 * invN) : rs * (a - xh * s2 * invN));
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    atomic_addv(dg + i, sacc[i]);
    if (KIND == 0) atomic_addv(db + i, sacc[N + i]);
  }
}

// Column sums of bf16 [M, N] (bias gradients): per-block partials [nb][N].
// A block covers `rows_per_block` rows; its threads are laid out as
// (N/8 column groups) x (256 / (N/8) row lanes) so every row is read with
// coalesced 16-byte loads, eight rows in flight per thread.
// blockIdx.y selects a slice of up to 2048 columns (rows longer than 2048 use several slices).
__global__ void __launch_bounds__(256) colsum_bf16_kernel(const __nv_bfloat16* __restrict__ dy,
                                                          float* __restrict__ part, int64_t M, int N,
                                                          int64_t rows_per_block, float* __restrict__ sum) {
  const int col0 = blockIdx.y * 2048;
  const int W = min(2048, N - col0);  // this slice's columns
  const int groups = W / 8;
  const int rpar = blockDim.x / groups;
  const int grp = threadIdx.x % groups, rl = threadIdx.x / groups;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_block;
  const int64_t r1 = r0 + rows_per_block < M ? r0 + rows_per_block : M;
  extern __shared__ float sc[];  // [rpar][W]
  dy += col0;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (rl < rpar) {
    int64_t r = r0 + rl;
    for (; r + 7 * rpar < r1; r += 8 * rpar) {
      uint4 u[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) u[k] = __ldg(reinterpret_cast<const uint4*>(dy + (r + k * rpar) * N + grp * 8));
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float2 a = unpack_bf16(u[k].x), b = unpack_bf16(u[k].y), c = unpack_bf16(u[k].z), d = unpack_bf16(u[k].w);
        acc[0] += a.x; acc[1] += a.y; acc[2] += b.x; acc[3] += b.y;
        acc[4] += c.x; acc[5] += c.y; acc[6] += d.x; acc[7] += d.y;
      }
    }
    for (; r < r1; r += rpar) {
      float v[8];
      load8(dy + r * N + grp * 8, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[rl * W + grp * 8 + j] = acc[j];
  }
  __syncthreads();
  // the block's column sums: a partial row, or (sum given, 16-byte aligned) added straight into sum
  if (sum) {
    for (int c = threadIdx.x * 4; c < W; c += blockDim.x * 4) {
      float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int k = 0; k < rpar; ++k) {
        const float4 v = *reinterpret_cast<const float4*>(sc + k * W + c);
        t.x += v.x; t.y += v.y; t.z += v.z; t.w += v.w;
      }
      atomicAdd(reinterpret_cast<float4*>(sum + col0 + c), t);
    }
    return;
  }
  for (int c = threadIdx.x; c < W; c += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < rpar; ++k) s += sc[k * W + c];
    part[(int64_t)blockIdx.x * N + col0 + c] = s;
  }
}

}  // namespace zl

// ================================================================== C ABI
using namespace zl;
#define ST(s) static_cast<cudaStream_t>(s)
static inline unsigned nblk(int64_t n, int t) { return (unsigned)((n + t - 1) / t); }
// True when any of the pointers is off a 16-byte boundary (the bf16 kernels move rows 16 bytes at a
// time; a misaligned vector access would fault the context, so the entry points refuse it instead).
static inline bool misaligned16(std::initializer_list<const void*> ps) {
  uintptr_t a = 0;
  for (const void* p : ps) a |= reinterpret_cast<uintptr_t>(p);
  return (a & 15) != 0;
}

extern "C" const char* zl_last_error(void) { return zl::g_err; }
extern "C" const char* zl_version(void) { return "zerollm_b200 0.1 (sm_100a)"; }

namespace zl {
int gemm_dev_error_read_and_clear();
int attn_tc_dev_error_read_and_clear();
}
extern "C" zl_status zl_device_error(int* code_out) {
  int v = zl::gemm_dev_error_read_and_clear();
  const int a = zl::attn_tc_dev_error_read_and_clear();
  if (!v) v = a;
  if (code_out) *code_out = v;
  return v ? set_error(ZL_ETIMEOUT, "device wait timed out (code %d)", v) : ZL_OK;
}

extern "C" zl_status zl_norm_forward_bf16(int kind, const zl_bf16* x, const float* gamma, const float* beta, zl_bf16* y,
                                          float* mean, float* rstd, int64_t M, int N, float eps, zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;
  if (N % 8 || N > 256 * kMaxRowChunks) return set_error(ZL_EUNSUPPORTED, "norm: N=%d must be a multiple of 8, <= 2048", N);
  if (kind == 0 && !beta) return set_error(ZL_EINVAL, "layernorm: beta is null");
  if (misaligned16({x, y})) return set_error(ZL_EINVAL, "norm: x and y must be 16-byte aligned");
  const auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  auto Y = reinterpret_cast<__nv_bfloat16*>(y);
  const int ch = N <= 256 ? 1 : N <= 512 ? 2 : N <= 1024 ? 4 : 8;
  // resident warps: 8 blocks of 8 warps per SM, each warp walks rows with the next one prefetched
  const int64_t nbf = std::min<int64_t>(nblk(M, 8), (int64_t)sm_count_current() * 8);
#define NF(K, C) norm_fwd_bf16_kernel<K, C><<<(unsigned)nbf, 256, 0, ST(s)>>>(X, gamma, K == 0 ? beta : nullptr, Y, K == 0 ? mean : nullptr, rstd, M, N, eps)
  if (kind == 0) { if (ch == 1) NF(0, 1); else if (ch == 2) NF(0, 2); else if (ch == 4) NF(0, 4); else NF(0, 8); }
  else { if (ch == 1) NF(1, 1); else if (ch == 2) NF(1, 2); else if (ch == 4) NF(1, 4); else NF(1, 8); }
#undef NF
  return check_launch("norm_fwd_bf16");
}
extern "C" int zl_norm_bwd_blocks(int64_t M) { return norm_bwd_blocks(M); }
namespace zl {
// Norm backward with optional column sums of dx (`dcol`, accumulated): the bias gradient of the
// layer whose output feeds this norm, so the model needs no separate column-sum pass for it.
// `workspace` holds nb * N * (1 + LayerNorm + (dcol != null)) floats.
zl_status norm_backward_bf16(int kind, const zl_bf16* x, const zl_bf16* dy, const float* gamma, const float* mean,
                             const float* rstd, zl_bf16* dx, float* dgamma, float* dbeta, float* dcol,
                             float* workspace, int64_t M, int N, cudaStream_t s, bool fused) {
  if (M <= 0 || N <= 0) return ZL_OK;
  if (N % 8 || N > 256 * kMaxRowChunks) return set_error(ZL_EUNSUPPORTED, "norm: N=%d must be a multiple of 8, <= 2048", N);
  // fused: every block adds its sums into dgamma / dbeta / dcol (16-byte atomics); otherwise block
  // partials go to the workspace and one fixed-order reduction follows
  fused = fused && !misaligned16({dgamma, dbeta, dcol});
  if ((!fused && !workspace) || !dgamma || (kind == 0 && (!dbeta || !mean)))
    return set_error(ZL_EINVAL, "norm bwd: null pointer");
  int nb = norm_bwd_blocks(M);
  const auto X = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto DY = reinterpret_cast<const __nv_bfloat16*>(dy);
  auto DX = reinterpret_cast<__nv_bfloat16*>(dx);
  const int NK = 1 + (kind == 0 ? 1 : 0) + (dcol ? 1 : 0);
  const size_t acc = (size_t)(N <= 512 ? 8 : 1) * NK * N * sizeof(float);
  const int ch = N <= 256 ? 1 : N <= 512 ? 2 : N <= 1024 ? 4 : 8;
  // rows stream through shared memory by bulk copy when x and dy are 16-byte aligned
  const bool staged = ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy)) & 15) == 0;
  const int stages = !staged ? 0 : ch <= 2 ? 3 : 2;
  // the staged kernel keeps two blocks resident per SM (one block for 2048 columns); one wave of
  // them, each warp with its rows in flight, beats more blocks
  if (stages > 0) nb = std::min(nb, sm_count_current() * (ch == 8 ? 1 : 2));
  const size_t sm = (size_t)8 * stages * 4 * N + (size_t)8 * stages * 8 + acc;
  // the partial sets dgamma | dbeta (LayerNorm) | column sums, in the kernel's order
  float* outs[3] = {dgamma, nullptr, nullptr};
  {
    int no = 1;
    if (kind == 0) outs[no++] = dbeta;
    if (dcol) outs[no++] = dcol;
  }
#define NB(K, C, COL, ST)                                                                                        \
  {                                                                                                              \
    auto kern = norm_bwd_bf16_kernel<K, C, COL, ST>;                                                             \
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);                            \
    kern<<<nb, 256, sm, s>>>(X, DY, gamma, K == 0 ? mean : nullptr, rstd, DX, fused ? nullptr : workspace, M, N, \
                             fused ? outs[0] : nullptr, outs[1], outs[2]);                                         \
  }
#define NBS(K, C, COL) { if (stages == 3) NB(K, C, COL, 3) else if (stages == 2) NB(K, C, COL, 2) else NB(K, C, COL, 0) }
#define NBC(K, COL) { if (ch == 1) NBS(K, 1, COL) else if (ch == 2) NBS(K, 2, COL) else if (ch == 4) NBS(K, 4, COL) else NBS(K, 8, COL) }
  if (kind == 0) { if (dcol) NBC(0, true) else NBC(0, false) }
  else { if (dcol) NBC(1, true) else NBC(1, false) }
#undef NBC
#undef NBS
#undef NB
  zl_status st = check_launch("norm_bwd_bf16");
  if (st != ZL_OK || fused) return st;
  // one reduction over the partial sets dgamma | dbeta (LayerNorm) | column sums
  launch_reduce_partials(workspace, nb, N, NK * N, outs[0], outs[1], s, outs[2]);
  return check_launch("norm_bwd_reduce");
}
}  // namespace zl
extern "C" zl_status zl_norm_backward_bf16(int kind, const zl_bf16* x, const zl_bf16* dy, const float* gamma,
                                           const float* mean, const float* rstd, zl_bf16* dx, float* dgamma,
                                           float* dbeta, float* workspace, int64_t M, int N, zl_stream s) {
  return zl::norm_backward_bf16(kind, x, dy, gamma, mean, rstd, dx, dgamma, dbeta, nullptr, workspace, M, N, ST(s),
                                false);
}

extern "C" zl_status zl_embedding_forward_bf16(const int32_t* ids, const float* table, const float* pos, zl_bf16* out,
                                               int64_t T, int seq_len, int dim, int vocab, zl_stream s) {
  if (T <= 0) return ZL_OK;
  if (dim % 8) return set_error(ZL_EUNSUPPORTED, "embedding: dim %% 8 != 0");
  if (misaligned16({table, pos, out})) return set_error(ZL_EINVAL, "embedding: table, pos and out must be 16-byte aligned");
  embed_fwd_bf16_kernel<<<nblk(T, 8), 256, 0, ST(s)>>>(ids, table, pos, reinterpret_cast<__nv_bfloat16*>(out), T,
                                                       seq_len, dim, vocab);
  return check_launch("embed_fwd_bf16");
}
extern "C" zl_status zl_embedding_backward_bf16(const int32_t* ids, const zl_bf16* dx, float* dtable, int64_t T, int dim,
                                                int vocab, zl_stream s) {
  if (T <= 0) return ZL_OK;
  if (dim % 8) return set_error(ZL_EUNSUPPORTED, "embedding: dim %% 8 != 0");
  if (misaligned16({dx, dtable})) return set_error(ZL_EINVAL, "embedding: dx and dtable must be 16-byte aligned");
  embed_bwd_bf16_kernel<<<nblk(T, 8), 256, 0, ST(s)>>>(ids, reinterpret_cast<const __nv_bfloat16*>(dx), dtable, T,
                                                       dim, vocab);
  return check_launch("embed_bwd_bf16");
}

extern "C" zl_status zl_cross_entropy_fused_bf16(zl_bf16* logits, const int32_t* targets, int rows, int vocab, float eps,
                                                 float grad_scale, float* loss_rows, float* loss_out, zl_stream s) {
  if (rows <= 0 || vocab <= 0) return set_error(ZL_EINVAL, "cross_entropy: sizes must be positive");
  if (vocab % 8) return set_error(ZL_EUNSUPPORTED, "cross_entropy: vocab %% 8 != 0");
  const size_t sm = (size_t)vocab * sizeof(float);
  auto lg = reinterpret_cast<__nv_bfloat16*>(logits);
  if (vocab <= 8 * 256 * 2) {
    ce_fused_reg_bf16_kernel<2><<<rows, 256, 0, ST(s)>>>(lg, targets, vocab, -logf(eps), grad_scale, loss_rows);
  } else if (vocab <= 8 * 256 * 4) {
    ce_fused_reg_bf16_kernel<4><<<rows, 256, 0, ST(s)>>>(lg, targets, vocab, -logf(eps), grad_scale, loss_rows);
  } else {
    if (sm > 200 * 1024) return set_error(ZL_EUNSUPPORTED, "cross_entropy: vocab too large");
    cudaFuncSetAttribute(ce_fused_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
    ce_fused_bf16_kernel<<<rows, 256, sm, ST(s)>>>(lg, targets, vocab, -logf(eps), grad_scale, loss_rows);
  }
  zl_status st = check_launch("ce_fused_bf16");
  if (st != ZL_OK || !loss_out) return st;
  mean_kernel<<<1, 1024, 0, ST(s)>>>(loss_rows, rows, loss_out, (float)rows);
  return check_launch("mean_kernel");
}

namespace {
// ~4 waves of 148 SMs x 2 resident blocks; at least 64 rows per block.
int64_t colsum_rows_per_block(int64_t M) {
  int64_t rpb = (M + 1183) / 1184;
  return rpb < 64 ? 64 : rpb;
}
}  // namespace
extern "C" int64_t zl_colsum_workspace_floats(int64_t M, int N) {
  const int64_t rpb = colsum_rows_per_block(M);
  return ((M + rpb - 1) / rpb) * N;
}
extern "C" zl_status zl_colsum_bf16(const zl_bf16* dy, float* db, float* workspace, int64_t M, int N, zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;
  if (N % 8) return set_error(ZL_EUNSUPPORTED, "colsum: N=%d must be a multiple of 8", N);
  if (misaligned16({dy})) return set_error(ZL_EINVAL, "colsum: dy must be 16-byte aligned");
  const int64_t rpb = colsum_rows_per_block(M);
  const int nb = (int)((M + rpb - 1) / rpb);
  const int slices = (N + 2047) / 2048;
  const int W = N < 2048 ? N : 2048;  // widest slice
  const int rpar = 256 / (W / 8);     // row lanes of the widest slice (narrower slices use more)
  const int smem_rows = 256 / ((N - (slices - 1) * 2048) / 8);
  const size_t smem = (size_t)std::max(rpar * W, smem_rows * (N - (slices - 1) * 2048)) * sizeof(float);
  colsum_bf16_kernel<<<dim3(nb, slices), 256, smem, ST(s)>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy), workspace, M, N, rpb, nullptr);
  zl_status st = check_launch("colsum_bf16");
  if (st != ZL_OK) return st;
  launch_reduce_partials(workspace, nb, N, N, db, nullptr, ST(s));
  return check_launch("colsum_reduce");
}

namespace zl {
// The model's bias-gradient column sums: each block adds its sums straight into db (16-byte fp32
// atomics, additions in any order), so there is no partial buffer and no second launch.
zl_status colsum_bf16_add(const zl_bf16* dy, float* db, int64_t M, int N, cudaStream_t s) {
  if (M <= 0 || N <= 0) return ZL_OK;
  if (N % 8) return set_error(ZL_EUNSUPPORTED, "colsum: N=%d must be a multiple of 8", N);
  if (misaligned16({dy, db})) return set_error(ZL_EINVAL, "colsum: dy and db must be 16-byte aligned");
  const int64_t rpb = colsum_rows_per_block(M);
  const int nb = (int)((M + rpb - 1) / rpb);
  const int slices = (N + 2047) / 2048;
  const int W = N < 2048 ? N : 2048;
  const int rpar = 256 / (W / 8);
  const int smem_rows = 256 / ((N - (slices - 1) * 2048) / 8);
  const size_t smem = (size_t)std::max(rpar * W, smem_rows * (N - (slices - 1) * 2048)) * sizeof(float);
  colsum_bf16_kernel<<<dim3(nb, slices), 256, smem, s>>>(reinterpret_cast<const __nv_bfloat16*>(dy), nullptr, M, N,
                                                           rpb, db);
  return check_launch("colsum_bf16");
}
}  // namespace zl

// ---------------------------------------------------------------- colsum without a caller workspace
// The partial sums of zl_colsum_bf16 live in this fixed device array instead of a caller buffer.
// Its device address is looked up once per device (cudaGetSymbolAddress) and kept; every partial
// is written by the column-sum kernel before the reduction reads it, so nothing needs clearing.
namespace {
constexpr int64_t kColsumScratchFloats = int64_t(1) << 20;  // 4 MiB
constexpr int kMaxDevices = 64;
static __device__ __align__(256) float colsum_scratch[kColsumScratchFloats];
std::mutex g_colsum_scratch_mu;
float* g_colsum_scratch_ptr[kMaxDevices] = {};

zl_status colsum_scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(ZL_ECUDA, "colsum_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(ZL_EUNSUPPORTED, "colsum_noalloc: device %d >= %d", dev, kMaxDevices);
  std::lock_guard<std::mutex> lock(g_colsum_scratch_mu);
  if (!g_colsum_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, colsum_scratch);
    if (e != cudaSuccess)
      return set_error(ZL_ECUDA, "colsum_noalloc: cudaGetSymbolAddress on device %d: %s", dev, cudaGetErrorString(e));
    g_colsum_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_colsum_scratch_ptr[dev];
  return ZL_OK;
}
}  // namespace

extern "C" int64_t zl_colsum_noalloc_max_floats(void) { return kColsumScratchFloats; }

extern "C" zl_status zl_colsum_bf16_noalloc(const zl_bf16* dy, float* db, int64_t M, int N, zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;
  if (N % 8) return set_error(ZL_EUNSUPPORTED, "colsum_noalloc: N=%d must be a multiple of 8", N);
  if (!dy || !db) return set_error(ZL_EINVAL, "colsum_noalloc: null pointer");
  if (misaligned16({dy})) return set_error(ZL_EINVAL, "colsum_noalloc: dy must be 16-byte aligned");
  const int64_t need = zl_colsum_workspace_floats(M, N);
  if (need > kColsumScratchFloats)
    return set_error(ZL_EINVAL,
                     "colsum_noalloc: M=%lld, N=%d needs %lld floats of scratch; the static maximum is %lld "
                     "(use zl_colsum_bf16 with a workspace)",
                     (long long)M, N, (long long)need, (long long)kColsumScratchFloats);
  float* scratch = nullptr;
  const zl_status st = colsum_scratch_for_current_device(&scratch);
  if (st != ZL_OK) return st;
  return zl_colsum_bf16(dy, db, scratch, M, N, s);
}

extern "C" zl_status zl_adamw_flat(float* params, const float* grads, float* m, float* v, zl_bf16* params_bf16, int64_t n,
                                   float lr, float weight_decay, float beta1, float beta2, float eps, float bc1,
                                   float bc2, float grad_scale, zl_stream s) {
  if (n <= 0) return set_error(ZL_EINVAL, "adamw: size must be > 0");
  adamw_kernel<<<nblk((n + 3) / 4, 256), 256, 0, ST(s)>>>(params, grads, m, v,
                                                         reinterpret_cast<__nv_bfloat16*>(params_bf16), n, lr,
                                                         weight_decay, beta1, beta2, eps, bc1, bc2, grad_scale);
  return check_launch("adamw_kernel");
}
extern "C" zl_status zl_f32_to_bf16(const float* x, zl_bf16* y, int64_t n, zl_stream s) {
  if (n <= 0) return ZL_OK;
  f32_to_bf16_kernel<<<nblk(n, 256), 256, 0, ST(s)>>>(x, reinterpret_cast<__nv_bfloat16*>(y), n);
  return check_launch("f32_to_bf16");
}

// ---------------------------------------------------------------- fp32 reference API
extern "C" zl_status zl_layernorm_forward_f32(const float* input, const float* gamma, const float* beta, float* output,
                                              float* mean, float* rstd, int64_t M, int64_t N, float eps, zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;  // layernorm.cu:178
  norm_fwd_f32_kernel<0, float><<<nblk(M, 8), 256, 0, ST(s)>>>(input, gamma, beta, output, mean, rstd, M, (int)N, eps);
  return check_launch("layernorm_forward_kernel");
}
extern "C" zl_status zl_layernorm_backward_f32(const float* input, const float* d_output, const float* gamma,
                                               const float* mean, const float* rstd, float* d_input, float* d_gamma,
                                               float* d_beta, int64_t M, int64_t N, zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;  // layernorm.cu:200
  const int nb = norm_bwd_blocks(M);
  norm_bwd_f32_kernel<0, float><<<nb, 256, 2 * N * sizeof(float), ST(s)>>>(input, d_output, gamma, mean, rstd, d_input,
                                                                    d_gamma, d_beta, M, (int)N);
  return check_launch("layernorm_backward_kernel");
}
extern "C" zl_status zl_rmsnorm_forward_f32(const float* input, const float* gamma, float* output, float* rstd, int64_t M,
                                            int64_t N, float eps, zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;
  norm_fwd_f32_kernel<1, float><<<nblk(M, 8), 256, 0, ST(s)>>>(input, gamma, nullptr, output, nullptr, rstd, M, (int)N, eps);
  return check_launch("rmsnorm_forward_kernel");
}
extern "C" zl_status zl_rmsnorm_backward_f32(const float* input, const float* d_output, const float* gamma,
                                             const float* rstd, float* d_input, float* d_gamma, int64_t M, int64_t N,
                                             zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;
  const int nb = norm_bwd_blocks(M);
  norm_bwd_f32_kernel<1, float><<<nb, 256, 2 * N * sizeof(float), ST(s)>>>(input, d_output, gamma, nullptr, rstd, d_input,
                                                                    d_gamma, nullptr, M, (int)N);
  return check_launch("rmsnorm_backward_kernel");
}
extern "C" zl_status zl_softmax_f32(const float* input, float* output, int M, int N, zl_stream s) {
  if (M <= 0 || N <= 0) return set_error(ZL_EINVAL, "softmax: M and N must be > 0");  // softmax.cu:70-71
  softmax_f32_kernel<<<M, 256, 0, ST(s)>>>(input, output, N);
  return check_launch("softmax_kernel");
}
extern "C" zl_status zl_cross_entropy_backward_f32(float* d_logits, const float* softmax_output, const int32_t* targets,
                                                   int batch, int num_classes, zl_stream s) {
  if (batch <= 0 || num_classes <= 0) return ZL_OK;  // cross_entropy.cu:39
  ce_bwd_f32_kernel<<<nblk((int64_t)batch * num_classes, 256), 256, 0, ST(s)>>>(d_logits, softmax_output, targets,
                                                                                batch, num_classes);
  return check_launch("cross_entropy_backward_kernel");
}
extern "C" zl_status zl_cross_entropy_forward_f32(const float* softmax_output, const int32_t* targets, int batch,
                                                  int num_classes, float eps, float* loss_out, zl_stream s) {
  if (batch <= 0 || num_classes <= 0)
    return set_error(ZL_EINVAL, "Batch size and number of classes must be positive");  // cross_entropy.cpp:26-28
  ce_loss_f32_kernel<<<1, 1024, 0, ST(s)>>>(softmax_output, targets, batch, num_classes, eps, loss_out);
  return check_launch("cross_entropy_forward");
}
extern "C" zl_status zl_embedding_forward_f32(const int32_t* input, const float* table, const float* pos, float* output,
                                              int batch, int seq_len, int embed_dim, int vocab_size, int max_seq_len,
                                              zl_stream s) {
  if (batch <= 0 || seq_len <= 0 || embed_dim <= 0) return ZL_OK;  // embedding.cu:66
  embed_fwd_f32_kernel<<<nblk((int64_t)batch * seq_len * embed_dim, 256), 256, 0, ST(s)>>>(
      input, table, pos, output, batch, seq_len, embed_dim, vocab_size, max_seq_len);
  return check_launch("embedding_forward_kernel");
}
extern "C" zl_status zl_embedding_backward_f32(const int32_t* input, const float* d_output, float* d_table, int batch,
                                               int seq_len, int embed_dim, int vocab_size, zl_stream s) {
  if (batch <= 0 || seq_len <= 0 || embed_dim <= 0) return ZL_OK;  // embedding.cu:87
  embed_bwd_f32_kernel<<<nblk((int64_t)batch * seq_len * embed_dim, 256), 256, 0, ST(s)>>>(
      input, d_output, d_table, batch, seq_len, embed_dim, vocab_size);
  return check_launch("embedding_backward_kernel");
}
extern "C" zl_status zl_add_f32(const float* a, const float* b, float* output, int size, zl_stream s) {
  if (size <= 0) return set_error(ZL_EINVAL, "add: size must be > 0");  // add.cu:36-38
  add_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(a, b, output, size);
  return check_launch("add_kernel");
}
extern "C" zl_status zl_add_inplace_f32(float* a, const float* b, int size, zl_stream s) {
  if (size <= 0) return set_error(ZL_EINVAL, "add_inplace: size must be > 0");
  add_inplace_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(a, b, size);
  return check_launch("add_inplace_kernel");
}
extern "C" zl_status zl_relu_forward_f32(const float* input, float* output, int size, zl_stream s) {
  if (size <= 0) return ZL_OK;  // relu.cu:23
  relu_fwd_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(input, output, size);
  return check_launch("relu_forward");
}
extern "C" zl_status zl_relu_backward_f32(const float* input, const float* grad_output, float* grad_input, int size,
                                          zl_stream s) {
  if (size <= 0) return ZL_OK;  // relu.cu:35
  relu_bwd_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(input, grad_output, grad_input, size);
  return check_launch("relu_backward");
}
extern "C" zl_status zl_transpose_f32(const float* input, float* output, int rows, int cols, zl_stream s) {
  if (rows <= 0 || cols <= 0) return ZL_OK;  // transpose.cu:19
  dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
  transpose_kernel<<<grid, block, 0, ST(s)>>>(input, output, rows, cols);
  return check_launch("transpose");
}
extern "C" zl_status zl_adamw_step_f32(float* params, const float* grads, float* m, float* v, int64_t size, float lr,
                                       float wd, float b1, float b2, float eps, float bc1, float bc2, zl_stream s) {
  if (size <= 0) return set_error(ZL_EINVAL, "adamw_step: size must be > 0");  // adamw.cu:92-94
  adamw_kernel<<<nblk((size + 3) / 4, 256), 256, 0, ST(s)>>>(params, grads, m, v, nullptr, size, lr, wd, b1, b2, eps,
                                                            bc1, bc2, 1.0f);
  return check_launch("adamw_kernel");
}
extern "C" zl_status zl_adam_step_f32(float* params, const float* grads, float* m, float* v, int64_t size, float lr,
                                      float b1, float b2, float eps, float bc1, float bc2, zl_stream s) {
  if (size <= 0) return set_error(ZL_EINVAL, "adam_step: size must be > 0");
  adam_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(params, grads, m, v, size, lr, b1, b2, eps, bc1, bc2);
  return check_launch("adam_kernel");
}
extern "C" zl_status zl_sgd_step_f32(float* params, const float* grads, float* velocity, int64_t size, float lr,
                                     float momentum, float weight_decay, zl_stream s) {
  if (size <= 0) return set_error(ZL_EINVAL, "sgd_step: size must be > 0");
  sgd_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(params, grads, velocity, size, lr, momentum, weight_decay);
  return check_launch("sgd_kernel");
}

// ---------------------------------------------------------------- bf16 instances of the reference API
// The reference instantiates these templates for float only; these are the __nv_bfloat16 instances
// (bf16 storage, fp32 arithmetic) with the same size checks and silent returns.
namespace {
inline const __nv_bfloat16* B16(const zl_bf16* p) { return reinterpret_cast<const __nv_bfloat16*>(p); }
inline __nv_bfloat16* B16(zl_bf16* p) { return reinterpret_cast<__nv_bfloat16*>(p); }
}  // namespace
extern "C" zl_status zl_layernorm_forward_bf16(const zl_bf16* input, const zl_bf16* gamma, const zl_bf16* beta,
                                               zl_bf16* output, zl_bf16* mean, zl_bf16* rstd, int64_t M, int64_t N,
                                               float eps, zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;  // layernorm.cu:178
  norm_fwd_f32_kernel<0, __nv_bfloat16><<<nblk(M, 8), 256, 0, ST(s)>>>(B16(input), B16(gamma), B16(beta), B16(output),
                                                                       B16(mean), B16(rstd), M, (int)N, eps);
  return check_launch("layernorm_forward_kernel");
}
extern "C" zl_status zl_layernorm_backward_bf16(const zl_bf16* input, const zl_bf16* d_output, const zl_bf16* gamma,
                                                const zl_bf16* mean, const zl_bf16* rstd, zl_bf16* d_input,
                                                zl_bf16* d_gamma, zl_bf16* d_beta, int64_t M, int64_t N, zl_stream s) {
  if (M <= 0 || N <= 0) return ZL_OK;  // layernorm.cu:200
  const int nb = norm_bwd_blocks(M);
  norm_bwd_f32_kernel<0, __nv_bfloat16><<<nb, 256, 2 * N * sizeof(float), ST(s)>>>(
      B16(input), B16(d_output), B16(gamma), B16(mean), B16(rstd), B16(d_input), B16(d_gamma), B16(d_beta), M, (int)N);
  return check_launch("layernorm_backward_kernel");
}
extern "C" zl_status zl_softmax_bf16(const zl_bf16* input, zl_bf16* output, int M, int N, zl_stream s) {
  if (M <= 0 || N <= 0) return set_error(ZL_EINVAL, "softmax: M and N must be > 0");  // softmax.cu:70-71
  softmax_f32_kernel<__nv_bfloat16><<<M, 256, 0, ST(s)>>>(B16(input), B16(output), N);
  return check_launch("softmax_kernel");
}
extern "C" zl_status zl_add_bf16(const zl_bf16* a, const zl_bf16* b, zl_bf16* output, int size, zl_stream s) {
  if (size <= 0) return set_error(ZL_EINVAL, "add: size must be > 0");  // add.cu:36-38
  add_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(B16(a), B16(b), B16(output), size);
  return check_launch("add_kernel");
}
extern "C" zl_status zl_add_inplace_bf16(zl_bf16* a, const zl_bf16* b, int size, zl_stream s) {
  if (size <= 0) return set_error(ZL_EINVAL, "add_inplace: size must be > 0");
  add_inplace_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(B16(a), B16(b), size);
  return check_launch("add_inplace_kernel");
}
extern "C" zl_status zl_relu_forward_bf16(const zl_bf16* input, zl_bf16* output, int size, zl_stream s) {
  if (size <= 0) return ZL_OK;  // relu.cu:23
  relu_fwd_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(B16(input), B16(output), size);
  return check_launch("relu_forward");
}
extern "C" zl_status zl_relu_backward_bf16(const zl_bf16* input, const zl_bf16* grad_output, zl_bf16* grad_input,
                                           int size, zl_stream s) {
  if (size <= 0) return ZL_OK;  // relu.cu:35
  relu_bwd_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(B16(input), B16(grad_output), B16(grad_input), size);
  return check_launch("relu_backward");
}
extern "C" zl_status zl_adamw_step_bf16(zl_bf16* params, const zl_bf16* grads, zl_bf16* m, zl_bf16* v, int64_t size,
                                        float lr, float wd, float b1, float b2, float eps, float bc1, float bc2,
                                        zl_stream s) {
  if (size <= 0) return set_error(ZL_EINVAL, "adamw_step: size must be > 0");  // adamw.cu:92-94
  adamw_bf16_kernel<<<nblk(size, 256), 256, 0, ST(s)>>>(B16(params), B16(grads), B16(m), B16(v), size, lr, wd, b1, b2,
                                                        eps, bc1, bc2);
  return check_launch("adamw_kernel");
}

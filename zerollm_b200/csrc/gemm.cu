// gemm.cu -- tcgen05 / TMEM / TMA GEMM for sm_100a with fused epilogues.
//
// Replaces the reference's SIMT GEMMs (src/kernel/cuda/matmul.cu:51-218,
// linear.cu:72-170) on the training path.  One persistent kernel computes
//     D[M,N] = sum_k A(m,k) * B(n,k)
// where A is stored K-major ([M,K]) or MN-major ([K,M]) and likewise B, so
// the forward (X W^T), input-gradient (dY W) and weight-gradient (dY^T X)
// products are all the same kernel with different operand majorness -- no
// transposes through HBM.
//
// CTA = 10 warps: warp 0 issues TMA loads into a STAGES-deep shared-memory
// ring (128-byte swizzle), warp 1 owns TMEM and issues tcgen05.mma from one
// thread into one of two 128 x BN fp32 accumulators, warps 2-9 (two per TMEM
// lane quarter) drain the other accumulator (tcgen05.ld) through the fused
// epilogue and store it by TMA.
// Every wait is bounded (common.cuh); a timeout records an error and the CTA
// unwinds, freeing TMEM.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "common.cuh"

namespace zl {

// ------------------------------------------------------------------ config
constexpr int BM = 128;
constexpr int kEpiWarps = 8;                       // two warps per TMEM lane quarter
constexpr int kThreads = 64 + kEpiWarps * 32;      // producer warp + MMA warp + epilogue
constexpr int kStgStride = 80;                     // bytes per staged row: 64 B of data + 16 B pad
constexpr int kStgBytes = 4096;                    // per epilogue warp: a 32 x 32 fp32 tile for the TMA store
static_assert(32 * kStgStride <= kStgBytes, "staging");

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static constexpr int bytes = 2, BK = 64, UMMA_K = 16, fmt = 1;
};
template <>
struct Elem<float> {
  static constexpr int bytes = 4, BK = 32, UMMA_K = 8, fmt = 2;
};

struct GemmArgs {
  int M, N, K;
  int n_tiles_n, tiles, k_blocks, splits, kb_per_split, units;
  int tma_out;  // full chunks leave through TMA stores (tensor maps of D and of the split-K workspace)
  int split_direct;  // accumulating fp32 output: every split adds its partial into D (TMA reduce-add)
  void* D;
  int flags;
  zl_epilogue epi;
  float* ws;  // split-K partials [splits][M][N] (fp32) when splits > 1
  float* colsum;  // when set (bf16 epilogue kinds only): column sums of the stored output added here
  // ReLU masks as bits ([M][N/32] words, bit j of word w = column 32 w + j): bits_out (when set, bf16
  // epilogue kinds) receives (stored value > 0) of every output; bits_in is the EK_MASKBITS kind's mask
  uint32_t* bits_out;
  const uint32_t* bits_in;
  int* sched;  // the run-time unit counter, or null for round-robin units
};

template <int BN, int STAGES, int ELEM_BYTES>
struct Smem {
  static constexpr int A_BYTES = BM * 128;   // BM rows (or BK rows x BM) of 128 bytes
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;            // per-warp staging for coalesced epilogue I/O
  static constexpr int BAR_OFF = EPI_OFF + kEpiWarps * kStgBytes;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;  // barriers + alignment slack
};

// ------------------------------------------------------------------ work units
// A persistent CTA (or CTA pair) walks output tiles (x split-K slices) as work units.  Its first
// unit is its own index (the grid never exceeds the unit count), known to every role.  With
// args.sched set, each later one is drawn at run time: the number of CTAs (pairs) plus the next
// value of the counter *sched.  Units still start in index order, but a CTA that starts late,
// because another kernel still holds its SM (an all-reduce on a side stream), takes fewer of them
// instead of holding back the end of the launch.  Every drawing CTA draws until it gets a value at
// or past the unit count (its end marker) and then stops, so a launch draws exactly `units` values;
// the CTA that draws the last one puts the counter back to zero.  Consecutive launches in one stream
// can therefore share it; launches that may run at the same time must not.  Without sched the units
// go round-robin over the CTAs, and no role touches the ring (measured: the ring's hand-offs alone
// cost the bf16-epilogue products 2-8 %).  The TMA thread (of the even CTA, in a pair) draws each
// unit one unit ahead, so the counter's round trip overlaps a unit's loads, and publishes the CTA's
// units after the first in a ring of UNIT_RING shared-memory slots, which every other role reads
// once each, in order (ring position k - 1 holds the CTA's k-th unit).
constexpr int UNIT_RING = 4;
__device__ __forceinline__ int unit_draw(const GemmArgs& a, int ctas) { return ctas + atomicAdd(a.sched, 1); }
// After the CTA's last draw (`drawn`, -1 if none): a CTA that stopped early, on a timed-out wait,
// draws on to its end marker, and the CTA that drew the launch's last value resets the counter.
__device__ __forceinline__ void unit_settle(const GemmArgs& a, int drawn, int ctas) {
  if (!a.sched) return;
  while (drawn < a.units) drawn = ctas + atomicAdd(a.sched, 1);
  if (drawn == ctas + a.units - 1) atomicExch(a.sched, 0);
}
// one-SM kernel: the TMA thread publishes; readers are whole warps
__device__ __forceinline__ bool unit_put(uint64_t* full, uint64_t* empty, volatile int* slot, int k, int u) {
  const int r = k % UNIT_RING;
  if (!bounded_wait(&empty[r], ((uint32_t)(k / UNIT_RING) & 1u) ^ 1u, DEV_TIMEOUT_UNIT)) return false;
  slot[r] = u;
  mbar_arrive(&full[r]);
  return true;
}
__device__ __forceinline__ int unit_get_warp(uint64_t* full, uint64_t* empty, volatile int* slot, int k) {
  const int r = k % UNIT_RING;
  if (!bounded_wait_warp(&full[r], (uint32_t)(k / UNIT_RING) & 1u, DEV_TIMEOUT_UNIT)) return -1;
  const int u = slot[r];
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[r]);
  return u;
}
// CTA pair: the even CTA's TMA thread writes the slot in both CTAs and arrives on both `full`
// barriers; the readers of both CTAs release the slot on the even CTA's `empty` barrier
__device__ __forceinline__ bool unit_put_pair(uint64_t* full, uint64_t* empty, volatile int* slot, int k, int u) {
  const int r = k % UNIT_RING;
  if (!bounded_wait_cluster(&empty[r], ((uint32_t)(k / UNIT_RING) & 1u) ^ 1u, DEV_TIMEOUT_UNIT)) return false;
  slot[r] = u;
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(mapa_shared(smem_u32((const void*)&slot[r]), 1)), "r"(u)
               : "memory");
  mbar_arrive(&full[r]);
  mbar_arrive_cluster(mapa_shared(smem_u32(&full[r]), 1));  // release: the store above is seen first
  return true;
}
// a whole warp (warp_wide) or a single thread reads the CTA's k-th unit; -1 when the wait timed out
__device__ __forceinline__ int unit_get_pair(uint64_t* full, uint64_t* empty, volatile int* slot, int k,
                                             bool warp_wide) {
  const int r = k % UNIT_RING;
  bool ok = bounded_wait_cluster(&full[r], (uint32_t)(k / UNIT_RING) & 1u, DEV_TIMEOUT_UNIT);
  if (warp_wide) ok = __all_sync(0xffffffffu, ok);
  if (!ok) return -1;
  const int u = slot[r];
  if (warp_wide) __syncwarp();
  if (!warp_wide || (threadIdx.x & 31) == 0) mbar_arrive_cluster(mapa_shared(smem_u32(&empty[r]), 0));
  return u;
}

// ------------------------------------------------------------------ epilogue
// Per-thread fused epilogue for 32 consecutive columns [c0, c0+32) of row r (used for
// partial chunks and by the split-K reduction).  Every loop is fully unrolled with a
// column predicate so the value array stays in registers.
__device__ __forceinline__ void epilogue_store32(const GemmArgs& a, int r, int c0, float (&v)[32]) {
  if (r >= a.M) return;
  const int f = a.flags;
  const int nvalid = min(32, a.N - c0);
  if (nvalid <= 0) return;
  const size_t rowoff = (size_t)r * a.N + c0;
  const int hd = a.epi.head_dim;
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < nvalid) {
      if (f & ZL_EPI_BIAS) v[j] += __ldg(a.epi.bias + c0 + j);
    }
  }
  if ((f & ZL_EPI_ROPE) && c0 < a.epi.rope_cols) {
    const int half = hd >> 1;
    const int pos = r % a.epi.rope_seq;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      if (j + 1 < nvalid && c0 + j < a.epi.rope_cols) {
        const int i = ((c0 + j) % hd) >> 1;
        const size_t ti = a.epi.rope_pair_major ? (size_t)i * a.epi.rope_seq + pos : (size_t)pos * half + i;
        const float c = __ldg(a.epi.rope_cos + ti), s = __ldg(a.epi.rope_sin + ti);
        const float x0 = v[j], x1 = v[j + 1];
        v[j] = x0 * c - x1 * s;
        v[j + 1] = x0 * s + x1 * c;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j < nvalid) {
      if (f & ZL_EPI_RESIDUAL)
        v[j] += __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.epi.residual)[rowoff + j]);
      if (f & ZL_EPI_RELU_MASK)
        v[j] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.epi.aux)[rowoff + j]) > 0.f ? v[j] : 0.f;
      if (f & ZL_EPI_RELU) v[j] = fmaxf(v[j], 0.f);
      if (f & ZL_EPI_OUT_F32) {
        float* out = reinterpret_cast<float*>(a.D) + rowoff + j;
        *out = (f & ZL_EPI_ACCUM) ? *out + v[j] : v[j];
      } else {
        reinterpret_cast<__nv_bfloat16*>(a.D)[rowoff + j] = __float2bfloat16_rn(v[j]);
      }
    }
  }
}

// ------------------------------------------------------------------ coalesced epilogue
// A warp owns 32 consecutive rows (one TMEM lane quarter) and walks 32-column
// chunks.  Row-wise data (residual / mask in, results out) moves between
// registers and global memory through a per-warp staging buffer in shared
// memory, so every global access instruction of the warp covers 8 full
// 64-byte row segments instead of 32 scattered 16-byte pieces.
__device__ __forceinline__ void stg_put_row(uint32_t stg, int lane, const uint4 (&u)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(stg + lane * kStgStride + q * 16), "r"(u[q].x),
                 "r"(u[q].y), "r"(u[q].z), "r"(u[q].w));
}
__device__ __forceinline__ void stg_get_row(uint32_t stg, int lane, uint4 (&u)[4]) {
#pragma unroll
  for (int q = 0; q < 4; ++q)
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(u[q].x), "=r"(u[q].y), "=r"(u[q].z), "=r"(u[q].w)
                 : "r"(stg + lane * kStgStride + q * 16));
}
// Global -> staging: 32 rows x 64 bytes starting at `base` (row pitch `pitch` bytes), rows < nrows.
__device__ __forceinline__ void stg_load(uint32_t stg, int lane, const uint8_t* base, size_t pitch, int nrows) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = i * 32 + lane, row = p >> 2, q = p & 3;
    uint4 u = make_uint4(0, 0, 0, 0);
    if (row < nrows) u = __ldg(reinterpret_cast<const uint4*>(base + (size_t)row * pitch + q * 16));
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(stg + row * kStgStride + q * 16), "r"(u.x), "r"(u.y),
                 "r"(u.z), "r"(u.w));
  }
}
// Staging -> global, same geometry.
__device__ __forceinline__ void stg_store(uint32_t stg, int lane, uint8_t* base, size_t pitch, int nrows) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = i * 32 + lane, row = p >> 2, q = p & 3;
    uint4 u;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                 : "r"(stg + row * kStgStride + q * 16));
    if (row < nrows) *reinterpret_cast<uint4*>(base + (size_t)row * pitch + q * 16) = u;
  }
}
__device__ __forceinline__ void unpack8(const uint4& u, float* v) {
  float2 a = unpack_bf16(u.x), b = unpack_bf16(u.y), c = unpack_bf16(u.z), d = unpack_bf16(u.w);
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y; v[4] = c.x; v[5] = c.y; v[6] = d.x; v[7] = d.y;
}

// Fused epilogue for one 32 x 32 chunk: rows [r0, r0+32) (this lane: r0+lane), columns [c0, c0+32).
// Requires N % 8 == 0 (bf16 out) / N % 4 == 0 (fp32 out) and c0 + 32 <= N; other chunks use
// epilogue_store32 (per-thread path).
// The warp's 32 x 32 chunk (this lane: row `lane`) as a swizzled tile in its staging buffer, then one
// TMA store (or element-wise add for an accumulating fp32 output) of the box at (c0, r0).
// bf16: rows of 64 bytes, 64-byte swizzle; fp32: rows of 128 bytes, 128-byte swizzle.  The
// buffer is 1024-byte aligned and its previous bulk copy has finished reading it.
__device__ __forceinline__ void chunk_tma_out(const CUtensorMap* tm, uint32_t stg, int lane, int r0, int c0,
                                              const float (&v)[32], bool f32, bool add) {
  if (f32) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t dst = stg + lane * 128 + ((q ^ (lane & 7)) << 4);
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(__float_as_uint(v[q * 4])),
                   "r"(__float_as_uint(v[q * 4 + 1])), "r"(__float_as_uint(v[q * 4 + 2])),
                   "r"(__float_as_uint(v[q * 4 + 3])));
    }
  } else {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t dst = stg + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4);
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(pack_bf16(v[q * 8 + 0], v[q * 8 + 1])),
                   "r"(pack_bf16(v[q * 8 + 2], v[q * 8 + 3])), "r"(pack_bf16(v[q * 8 + 4], v[q * 8 + 5])),
                   "r"(pack_bf16(v[q * 8 + 6], v[q * 8 + 7])));
    }
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (add) tma_reduce_add_2d_bulk(tm, stg, c0, r0);
    else tma_store_2d_bulk(tm, stg, c0, r0);
    bulk_commit();
  }
}

// Before the staging buffer is written again: the lane that issued the last bulk copy waits until
// that copy has read it.
__device__ __forceinline__ void stg_reclaim(int lane) {
  if (lane == 0) bulk_wait_read0();
  __syncwarp();
}

__device__ __forceinline__ void epilogue_chunk(const GemmArgs& a, uint32_t stg, int lane, int r0, int c0,
                                               float (&v)[32], const CUtensorMap* tm_out = nullptr) {
  int f = a.flags;
  const int r = r0 + lane;
  const int nrows = min(32, a.M - r0);
  if (f & ZL_EPI_BIAS) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = __ldg(reinterpret_cast<const float4*>(a.epi.bias + c0) + q);
      v[q * 4] += b.x; v[q * 4 + 1] += b.y; v[q * 4 + 2] += b.z; v[q * 4 + 3] += b.w;
    }
  }
  if ((f & ZL_EPI_ROPE) && c0 < a.epi.rope_cols) {
    const int half = a.epi.head_dim >> 1;
    const int pos = r % a.epi.rope_seq;
    // element i of this row's table slice: pair-major tables are [half, seq]
    const size_t t0 = a.epi.rope_pair_major ? (size_t)pos : (size_t)pos * half;
    const size_t ts = a.epi.rope_pair_major ? (size_t)a.epi.rope_seq : 1;
    const int i0 = (c0 % a.epi.head_dim) >> 1;
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      const size_t ti = t0 + (size_t)(i0 + (j >> 1)) * ts;
      const float c = __ldg(a.epi.rope_cos + ti), s = __ldg(a.epi.rope_sin + ti);
      const float x0 = v[j], x1 = v[j + 1];
      v[j] = x0 * c - x1 * s;
      v[j + 1] = x0 * s + x1 * c;
    }
  }
  if (tm_out) {
    // TMA-store path: the staging buffer belongs to the output tile, so residual and mask row
    // segments (64 contiguous bytes per lane) are read straight into registers; residual first,
    // then the mask, as below
#pragma unroll
    for (int pass = 0; pass < 2; ++pass) {
      const int flag = pass == 0 ? ZL_EPI_RESIDUAL : ZL_EPI_RELU_MASK;
      if (!(f & flag)) continue;
      const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(pass == 0 ? a.epi.residual : a.epi.aux);
      uint4 u[4] = {};
      if (r < a.M) {
        const uint4* p = reinterpret_cast<const uint4*>(src + (size_t)r * a.N + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) u[q] = __ldg(p + q);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float t[8];
        unpack8(u[q], t);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          if (pass == 0) v[q * 8 + k] += t[k];
          else v[q * 8 + k] = t[k] > 0.f ? v[q * 8 + k] : 0.f;
        }
      }
    }
    f &= ~(ZL_EPI_RESIDUAL | ZL_EPI_RELU_MASK);
  }
  if (f & ZL_EPI_RESIDUAL) {
    __syncwarp();
    stg_load(stg, lane, reinterpret_cast<const uint8_t*>(reinterpret_cast<const __nv_bfloat16*>(a.epi.residual) +
                                                         (size_t)r0 * a.N + c0),
             (size_t)a.N * 2, nrows);
    __syncwarp();
    uint4 u[4];
    stg_get_row(stg, lane, u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float t[8];
      unpack8(u[q], t);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[q * 8 + k] += t[k];
    }
  }
  if (f & ZL_EPI_RELU_MASK) {
    __syncwarp();
    stg_load(stg, lane, reinterpret_cast<const uint8_t*>(reinterpret_cast<const __nv_bfloat16*>(a.epi.aux) +
                                                         (size_t)r0 * a.N + c0),
             (size_t)a.N * 2, nrows);
    __syncwarp();
    uint4 u[4];
    stg_get_row(stg, lane, u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float t[8];
      unpack8(u[q], t);
#pragma unroll
      for (int k = 0; k < 8; ++k) v[q * 8 + k] = t[k] > 0.f ? v[q * 8 + k] : 0.f;
    }
  }
  if (f & ZL_EPI_RELU) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
  }
  if (tm_out) {
    __syncwarp();  // the residual / mask rows in the buffer have been read
    const bool f32 = (f & ZL_EPI_OUT_F32) != 0;
    chunk_tma_out(tm_out, stg, lane, r0, c0, v, f32, f32 && (f & ZL_EPI_ACCUM) != 0);
    return;
  }
  if (f & ZL_EPI_OUT_F32) {
    float* out = reinterpret_cast<float*>(a.D) + (size_t)r0 * a.N + c0;
    const bool acc = (f & ZL_EPI_ACCUM) != 0;
#pragma unroll
    for (int h = 0; h < 2; ++h) {  // 16 fp32 columns = 64 bytes per staged row
      if (acc) {
        __syncwarp();
        stg_load(stg, lane, reinterpret_cast<const uint8_t*>(out + h * 16), (size_t)a.N * 4, nrows);
        __syncwarp();
        uint4 u[4];
        stg_get_row(stg, lane, u);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          v[h * 16 + q * 4 + 0] += __uint_as_float(u[q].x);
          v[h * 16 + q * 4 + 1] += __uint_as_float(u[q].y);
          v[h * 16 + q * 4 + 2] += __uint_as_float(u[q].z);
          v[h * 16 + q * 4 + 3] += __uint_as_float(u[q].w);
        }
      }
      uint4 u[4];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        u[q] = make_uint4(__float_as_uint(v[h * 16 + q * 4]), __float_as_uint(v[h * 16 + q * 4 + 1]),
                          __float_as_uint(v[h * 16 + q * 4 + 2]), __float_as_uint(v[h * 16 + q * 4 + 3]));
      __syncwarp();
      stg_put_row(stg, lane, u);
      __syncwarp();
      stg_store(stg, lane, reinterpret_cast<uint8_t*>(out + h * 16), (size_t)a.N * 4, nrows);
    }
  } else {
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.D) + (size_t)r0 * a.N + c0;
    uint4 u[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      u[q].x = pack_bf16(v[q * 8 + 0], v[q * 8 + 1]);
      u[q].y = pack_bf16(v[q * 8 + 2], v[q * 8 + 3]);
      u[q].z = pack_bf16(v[q * 8 + 4], v[q * 8 + 5]);
      u[q].w = pack_bf16(v[q * 8 + 6], v[q * 8 + 7]);
    }
    __syncwarp();
    stg_put_row(stg, lane, u);
    __syncwarp();
    stg_store(stg, lane, reinterpret_cast<uint8_t*>(out), (size_t)a.N * 2, nrows);
  }
}

// Split-K partial chunk: raw fp32 accumulators to ws[split] (coalesced through staging).
__device__ __forceinline__ void partial_chunk(const GemmArgs& a, uint32_t stg, int lane, int split, int r0, int c0,
                                              const float (&v)[32], const CUtensorMap* tm_ws = nullptr) {
  if (tm_ws) {  // ws viewed as [splits * M, N]
    chunk_tma_out(tm_ws, stg, lane, split * a.M + r0, c0, v, true, false);
    return;
  }
  const int nrows = min(32, a.M - r0);
  float* out = a.ws + ((size_t)split * a.M + r0) * a.N + c0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    uint4 u[4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
      u[q] = make_uint4(__float_as_uint(v[h * 16 + q * 4]), __float_as_uint(v[h * 16 + q * 4 + 1]),
                        __float_as_uint(v[h * 16 + q * 4 + 2]), __float_as_uint(v[h * 16 + q * 4 + 3]));
    __syncwarp();
    stg_put_row(stg, lane, u);
    __syncwarp();
    stg_store(stg, lane, reinterpret_cast<uint8_t*>(out + h * 16), (size_t)a.N * 4, nrows);
  }
}

// ------------------------------------------------------------------ pipelined bf16 epilogue
// One epilogue warp's share of an accumulator tile with a bf16 output leaving by TMA store: rows
// [r0, r0+32) (this lane: r0+lane), columns n0 + [cbase, cbase + BN/2) in 32-column chunks.  The
// global inputs of chunk k+1 (bias column, residual or mask rows, RoPE table entries) are loaded
// while chunk k is finished, and two 2 KB staging boxes alternate, so a chunk never waits for the
// previous chunk's store to read its box.  KIND fixes which row-wise input the chunk reads, so
// that only its prefetch registers exist; bias and ReLU are runtime flags.
enum EpiKind : int { EK_PLAIN = 0, EK_RESIDUAL = 1, EK_MASK = 2, EK_ROPE = 3, EK_MASKBITS = 4 };

template <int KIND>
struct EpiPrefetch {
  float bias = 0.f;  // lane j: bias of column c0 + j
  uint4 row[(KIND == EK_RESIDUAL || KIND == EK_MASK) ? 4 : 1];  // residual / mask row segment (64 bytes)
  uint32_t mword = 0;                       // EK_MASKBITS: this row's mask bits of the chunk's 32 columns
  float rc[KIND == EK_ROPE ? 16 : 1], rs[KIND == EK_ROPE ? 16 : 1];  // cos / sin of 16 pairs
};

template <int KIND>
__device__ __forceinline__ void epi_fetch(const GemmArgs& a, int r, int lane, int c0, EpiPrefetch<KIND>& p) {
  if (a.flags & ZL_EPI_BIAS) p.bias = __ldg(a.epi.bias + c0 + lane);
  if constexpr (KIND == EK_RESIDUAL || KIND == EK_MASK) {
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(KIND == EK_RESIDUAL ? a.epi.residual : a.epi.aux);
#pragma unroll
    for (int q = 0; q < 4; ++q) p.row[q] = make_uint4(0, 0, 0, 0);
    if (r < a.M) {
      const uint4* s = reinterpret_cast<const uint4*>(src + (size_t)r * a.N + c0);
#pragma unroll
      for (int q = 0; q < 4; ++q) p.row[q] = __ldg(s + q);
    }
  }
  if constexpr (KIND == EK_MASKBITS) p.mword = r < a.M ? __ldg(a.bits_in + (size_t)r * (a.N >> 5) + (c0 >> 5)) : 0u;
  if constexpr (KIND == EK_ROPE) {
    if (c0 < a.epi.rope_cols) {
      const int half = a.epi.head_dim >> 1, i0 = (c0 % a.epi.head_dim) >> 1, pos = r % a.epi.rope_seq;
      if (a.epi.rope_pair_major) {  // [half, seq]: the warp's 32 positions are one 128-byte line per pair
        const size_t base = (size_t)i0 * a.epi.rope_seq + pos;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          p.rc[j] = __ldg(a.epi.rope_cos + base + (size_t)j * a.epi.rope_seq);
          p.rs[j] = __ldg(a.epi.rope_sin + base + (size_t)j * a.epi.rope_seq);
        }
      } else {  // [seq, half]: 64 contiguous bytes of this lane's row
        const size_t base = (size_t)pos * half + i0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 c4 = __ldg(reinterpret_cast<const float4*>(a.epi.rope_cos + base) + q);
          const float4 s4 = __ldg(reinterpret_cast<const float4*>(a.epi.rope_sin + base) + q);
          p.rc[4 * q] = c4.x; p.rc[4 * q + 1] = c4.y; p.rc[4 * q + 2] = c4.z; p.rc[4 * q + 3] = c4.w;
          p.rs[4 * q] = s4.x; p.rs[4 * q + 1] = s4.y; p.rs[4 * q + 2] = s4.z; p.rs[4 * q + 3] = s4.w;
        }
      }
    }
  }
}

// Before a tile's accumulator is ready: pull this lane's row segment of the residual or mask
// input for the warp's BN/2 columns into L2, so that the per-chunk loads (issued one chunk ahead)
// find it there instead of waiting on HBM.
template <int BN, int KIND>
__device__ __forceinline__ void epi_prefetch_l2(const GemmArgs& a, int r, int c0) {
  if constexpr (KIND == EK_RESIDUAL || KIND == EK_MASK) {
    if (r >= a.M || c0 >= a.N) return;
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(KIND == EK_RESIDUAL ? a.epi.residual : a.epi.aux);
    const char* p = reinterpret_cast<const char*>(src + (size_t)r * a.N + c0);
    const int bytes = min(BN / 2, a.N - c0) * 2;
    for (int o = 0; o < bytes; o += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(p + o));
  }
}

// Column sums of a warp's 32 x 32 output chunk added into dst[0, 32): lane l holds row l's values x[j]
// of columns j.  Five exchange steps (31 shuffles) halve the columns a lane keeps and sum them with the
// partner lane's, leaving lane j with the sum over all 32 rows of column j; one atomic add per lane.
__device__ __forceinline__ void chunk_colsum_add(float (&x)[32], int lane, float* dst) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool hi = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = hi ? x[i] : x[w + i];
      const float keep = hi ? x[w + i] : x[i];
      x[i] = keep + __shfl_xor_sync(0xffffffffu, send, w);
    }
  }
  atomicAdd(dst + lane, x[0]);
}

template <int BN, int KIND>
__device__ __forceinline__ void drain_bf16_tma(const GemmArgs& a, const CUtensorMap* tmD, uint32_t t_row,
                                               uint32_t stg, int lane, int r0, int n0, int cbase) {
  constexpr int NCH = BN / 64;
  const int f = a.flags;
  const int r = r0 + lane;
  EpiPrefetch<KIND> cur, nxt;
  epi_fetch<KIND>(a, r, lane, n0 + cbase, cur);
  uint32_t words[NCH];  // mask bits of this row's chunks (bits_out)
#pragma unroll
  for (int k = 0; k < NCH; ++k) words[k] = 0;
#pragma unroll 1
  for (int k = 0; k < NCH; ++k) {
    const int c = cbase + k * 32, c0 = n0 + c;
    if (c0 >= a.N) break;
    uint32_t raw[32];
    tmem_ld32(t_row + (uint32_t)c, raw);
    if (k + 1 < NCH && c0 + 32 < a.N) epi_fetch<KIND>(a, r, lane, c0 + 32, nxt);
    tmem_ld_wait();
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
    if (f & ZL_EPI_BIAS) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += __shfl_sync(0xffffffffu, cur.bias, j);
    }
    if constexpr (KIND == EK_ROPE) {
      if (c0 < a.epi.rope_cols) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float x0 = v[2 * j], x1 = v[2 * j + 1];
          v[2 * j] = x0 * cur.rc[j] - x1 * cur.rs[j];
          v[2 * j + 1] = x0 * cur.rs[j] + x1 * cur.rc[j];
        }
      }
    }
    if constexpr (KIND == EK_MASKBITS) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = ((cur.mword >> j) & 1u) ? v[j] : 0.f;
    }
    if constexpr (KIND == EK_RESIDUAL || KIND == EK_MASK) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float t[8];
        unpack8(cur.row[q], t);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (KIND == EK_RESIDUAL) v[q * 8 + j] += t[j];
          else v[q * 8 + j] = t[j] > 0.f ? v[q * 8 + j] : 0.f;
        }
      }
    }
    if (f & ZL_EPI_RELU) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
    }
    uint32_t pk[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) pk[j] = pack_bf16(v[2 * j], v[2 * j + 1]);
    if (a.bits_out) {  // bit j: the stored bf16 value of column c0 + j is > 0
      uint32_t word = 0;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        word |= ((int16_t)(pk[j] & 0xffffu) > 0 ? 1u : 0u) << (2 * j);
        word |= ((int16_t)(pk[j] >> 16) > 0 ? 1u : 0u) << (2 * j + 1);
      }
#pragma unroll
      for (int kk = 0; kk < NCH; ++kk)
        if (kk == k) words[kk] = word;  // register-resident: the index is a compile-time constant
      if (n0 + cbase + NCH * 32 > a.N && r < a.M)  // a partial warp slice: one word at a time
        a.bits_out[(size_t)r * (a.N >> 5) + (c0 >> 5)] = word;
    }
    // stage [32][32] bf16 (64-byte swizzle) in box k & 1, whose store from chunk k-2 has read it
    const uint32_t box = stg + (uint32_t)((k & 1) * 2048);
    if (lane == 0) bulk_wait_read1();
    __syncwarp();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t dst = box + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4);
      asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(dst), "r"(pk[q * 4]), "r"(pk[q * 4 + 1]),
                   "r"(pk[q * 4 + 2]), "r"(pk[q * 4 + 3]));
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d_bulk(tmD, box, c0, r0);
      bulk_commit();
    }
    if (a.colsum) {  // column sums of the stored (bf16-rounded) values; rows past M count as zero
      const bool in = r < a.M;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        v[2 * j] = in ? __uint_as_float(pk[j] << 16) : 0.f;
        v[2 * j + 1] = in ? __uint_as_float(pk[j] & 0xffff0000u) : 0.f;
      }
      chunk_colsum_add(v, lane, a.colsum + c0);
    }
    cur = nxt;
  }
  // the warp's whole slice of the row's mask words in 16-byte stores (the other column half's warp
  // writes the neighbouring 16 bytes of the same row)
  if (a.bits_out && r < a.M && n0 + cbase + NCH * 32 <= a.N) {
    uint32_t* dst = a.bits_out + (size_t)r * (a.N >> 5) + ((n0 + cbase) >> 5);
    static_assert(NCH % 2 == 0, "mask words go out in pairs or quadruples");
    if constexpr (NCH % 4 == 0) {
#pragma unroll
      for (int k = 0; k < NCH; k += 4)
        *reinterpret_cast<uint4*>(dst + k) = make_uint4(words[k], words[k + 1], words[k + 2], words[k + 3]);
    } else {
#pragma unroll
      for (int k = 0; k < NCH; k += 2) *reinterpret_cast<uint2*>(dst + k) = make_uint2(words[k], words[k + 1]);
    }
  }
}

// The kind of the pipelined bf16 epilogue for these flags, or -1 when the general path is needed
// (fp32 output, split-K partials, two row-wise inputs at once, or chunks that are not whole).
__host__ __device__ inline int bf16_epi_kind(int flags, int N, int splits) {
  if ((flags & (ZL_EPI_OUT_F32 | ZL_EPI_ACCUM)) || splits > 1 || N % 32 != 0) return -1;
  const int rows = (flags & ZL_EPI_RESIDUAL ? 1 : 0) + (flags & ZL_EPI_RELU_MASK ? 1 : 0) + (flags & ZL_EPI_ROPE ? 1 : 0);
  if (rows > 1) return -1;
  if (flags & ZL_EPI_RESIDUAL) return EK_RESIDUAL;
  if (flags & ZL_EPI_RELU_MASK) return EK_MASK;
  if (flags & ZL_EPI_ROPE) return EK_ROPE;
  return EK_PLAIN;
}

// ------------------------------------------------------------------ kernel
template <typename T, int BN, int STAGES, bool A_MN, bool B_MN, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmW,
                   const GemmArgs args) {
  using E = Elem<T>;
  using L = Smem<BN, STAGES, E::bytes>;
  constexpr int BK = E::BK;
  constexpr int ATOM = 128 / E::bytes;        // elements per 128-byte row
  constexpr uint32_t TMEM_COLS = 2 * BN;      // two accumulators
  constexpr uint32_t IDESC = make_idesc(E::fmt, BM, BN, A_MN ? 1u : 0u, B_MN ? 1u : 0u);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
  uint64_t* u_full = acc_empty + 3;  // [UNIT_RING] the work-unit ring
  uint64_t* u_empty = u_full + UNIT_RING;
  volatile int* u_slot = reinterpret_cast<volatile int*>(u_empty + UNIT_RING);
  static_assert((2 * STAGES + 5 + 2 * UNIT_RING) * 8 + UNIT_RING * 4 <= 256, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], kEpiWarps * 32); }
    for (int i = 0; i < UNIT_RING; ++i) { mbar_init(&u_full[i], 1); mbar_init(&u_empty[i], 1 + kEpiWarps); }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int u = (int)blockIdx.x, drawn = -1;
      for (int ku = 0; ok; ++ku) {
        if (args.sched && ku > 0 && !unit_put(u_full, u_empty, u_slot, ku - 1, u)) break;
        if (u >= args.units) break;
        const int u_next = args.sched ? unit_draw(args, (int)gridDim.x) : u + (int)gridDim.x;
        drawn = u_next;
        const int tile = u / args.splits, split = u % args.splits;
        const int m0 = (tile / args.n_tiles_n) * BM, n0 = (tile % args.n_tiles_n) * BN;
        const int kb0 = split * args.kb_per_split;
        const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!bounded_wait(&empty[stage], phase ^ 1u, DEV_TIMEOUT_EMPTY)) { ok = false; break; }
          uint8_t* sA = smem + stage * L::STAGE_BYTES;
          uint8_t* sB = sA + L::A_BYTES;
          mbar_arrive_expect_tx(&full[stage], L::STAGE_BYTES);
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d(sA, &tmA, &full[stage], k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < BM / ATOM; ++c) tma_load_2d(sA + c * BK * 128, &tmA, &full[stage], m0 + c * ATOM, k0);
          }
          if (!B_MN) {
            tma_load_2d(sB, &tmB, &full[stage], k0, n0);
          } else {
#pragma unroll
            for (int c = 0; c < BN / ATOM; ++c) tma_load_2d(sB + c * BK * 128, &tmB, &full[stage], n0 + c * ATOM, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        u = u_next;
      }
      unit_settle(args, drawn, (int)gridDim.x);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer
    int stage = 0;
    uint32_t phase = 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    bool ok = true;
    for (int ku = 0; ok; ++ku) {
      const int u = (ku == 0 || !args.sched) ? (int)blockIdx.x + ku * (int)gridDim.x
                                             : unit_get_warp(u_full, u_empty, u_slot, ku - 1);
      if (u < 0 || u >= args.units) break;
      const int split = u % args.splits;
      const int kb0 = split * args.kb_per_split;
      const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
      if (!bounded_wait(&acc_empty[acc], acc_phase ^ 1u, DEV_TIMEOUT_ACC)) { ok = false; break; }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!bounded_wait(&full[stage], phase, DEV_TIMEOUT_FULL)) { ok = false; break; }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_base = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t b_base = a_base + L::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / E::UMMA_K; ++k) {
            uint64_t ad, bd;
            if (!A_MN) ad = smem_desc_sw128(a_base + k * E::UMMA_K * E::bytes, 16, 1024);
            else       ad = smem_desc_sw128(a_base + k * E::UMMA_K * 128, BK * 128, 1024);
            if (!B_MN) bd = smem_desc_sw128(b_base + k * E::UMMA_K * E::bytes, 16, 1024);
            else       bd = smem_desc_sw128(b_base + k * E::UMMA_K * 128, BK * 128, 1024);
            const uint32_t accumulate = (kb > kb0 || k > 0) ? 1u : 0u;
            if (E::fmt == 1) umma_f16(d_tmem, ad, bd, IDESC, accumulate);
            else             umma_tf32(d_tmem, ad, bd, IDESC, accumulate);
          }
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) { stage = 0; phase ^= 1u; }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&acc_full[acc]);
      __syncwarp();
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  } else {
    // ------------------------------------------------ epilogue (warps 2 .. 2+kEpiWarps)
    const int ew = warp - 2;
    const int quarter = warp & 3;            // TMEM lane quarter this warp may access
    const int col_half = ew >> 2;            // which half of the BN columns this warp drains
    const uint32_t stg = smem_u32(smem + L::EPI_OFF + ew * kStgBytes);
    const bool fast_ok = ((args.flags & ZL_EPI_OUT_F32) ? (args.N % 4 == 0) : (args.N % 8 == 0)) &&
                         (!(args.flags & ZL_EPI_ROPE) || args.epi.head_dim % 32 == 0);
    const bool use_tma = fast_ok && args.tma_out;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int ku = 0;; ++ku) {
      const int u = (ku == 0 || !args.sched) ? (int)blockIdx.x + ku * (int)gridDim.x
                                             : unit_get_warp(u_full, u_empty, u_slot, ku - 1);
      if (u < 0 || u >= args.units) break;
      const int tile = u / args.splits, split = u % args.splits;
      const int m0 = (tile / args.n_tiles_n) * BM, n0 = (tile % args.n_tiles_n) * BN;
      if constexpr (KIND >= 0) epi_prefetch_l2<BN, KIND>(args, m0 + quarter * 32 + lane, n0 + col_half * (BN / 2));
      if (!bounded_wait(&acc_full[acc], acc_phase, DEV_TIMEOUT_ACC)) break;
      tc_fence_after();
      const int r0 = m0 + quarter * 32;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      if constexpr (KIND >= 0) {  // bf16 output by TMA store, pipelined (the host chose KIND)
        if (r0 < args.M) drain_bf16_tma<BN, KIND>(args, &tmD, t_row, stg, lane, r0, n0, col_half * (BN / 2));
      } else
#pragma unroll 1
      for (int c = col_half * (BN / 2); c < (col_half + 1) * (BN / 2); c += 32) {
        uint32_t raw[32];
        tmem_ld32(t_row + (uint32_t)c, raw);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
        const int c0 = n0 + c;
        if (c0 >= args.N || r0 >= args.M) continue;
        const bool full_chunk = fast_ok && (c0 + 32 <= args.N);
        if (use_tma) stg_reclaim(lane);
        if (args.split_direct) {
          // every split adds its partial into D; the adds of different splits land in any order
          chunk_tma_out(&tmD, stg, lane, r0, c0, v, true, true);
        } else if (args.splits > 1) {
          // a box must not run past row M: the workspace map would carry it into the next split
          if (full_chunk) partial_chunk(args, stg, lane, split, r0, c0, v, (use_tma && r0 + 32 <= args.M) ? &tmW : nullptr);
          else if (r0 + lane < args.M) {
            float* out = args.ws + ((size_t)split * args.M + r0 + lane) * args.N + c0;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (c0 + j < args.N) out[j] = v[j];
          }
        } else if (full_chunk) {
          epilogue_chunk(args, stg, lane, r0, c0, v, use_tma ? &tmD : nullptr);
        } else {
          epilogue_store32(args, r0 + lane, c0, v);
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
    if (use_tma && lane == 0) bulk_wait0();  // this warp's output copies are complete
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------ two-SM GEMM (bf16)
// A cluster of two CTAs on two SMs computes 256 x BN output tiles with tcgen05.mma.cta_group::2:
// each CTA loads its own 128 rows of A and half of the BN columns of B (so every SM streams half
// of B per tile instead of all of it), the even CTA issues the MMAs for both, and each CTA keeps
// its 128 x BN half of the accumulator in its own TMEM and drains it with its own epilogue warps.
//   * full[s]      (even CTA) counts the bytes both CTAs' TMA loads bring into stage s
//   * empty[s]     (both CTAs) arrived by the MMA's multicast commit when stage s is consumed
//   * acc_full[b]  (both CTAs) arrived by the multicast commit when accumulator b is complete
//   * acc_empty[b] (even CTA) arrived by the epilogue threads of both CTAs
// No TMA load uses multicast.
template <int BN, int STAGES>
struct Smem2 {
  static constexpr int A_BYTES = BM * 128;         // this CTA's 128 rows of A (or BK x 128)
  static constexpr int B_BYTES = (BN / 2) * 128;   // this CTA's half of B
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int EPI_OFF = STAGES * STAGE_BYTES;
  static constexpr int BAR_OFF = EPI_OFF + kEpiWarps * kStgBytes;
  static constexpr int TOTAL = BAR_OFF + 256 + 1024;
};

template <int BN, int STAGES, bool A_MN, bool B_MN, int KIND>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmW,
                    const GemmArgs args) {
  using L = Smem2<BN, STAGES>;
  constexpr int BK = 64, UMMA_K = 16, ATOM = 64;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  constexpr uint32_t IDESC = make_idesc(1, 2 * BM, BN, A_MN ? 1u : 0u, B_MN ? 1u : 0u);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_empty + 2);
  uint64_t* u_full = acc_empty + 3;  // [UNIT_RING] the work-unit ring (the even CTA's `empty` counts)
  uint64_t* u_empty = u_full + UNIT_RING;
  volatile int* u_slot = reinterpret_cast<volatile int*>(u_empty + UNIT_RING);
  static_assert((2 * STAGES + 5 + 2 * UNIT_RING) * 8 + UNIT_RING * 4 <= 256, "barrier area");

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = (int)blockIdx.x >> 1, npairs = (int)gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
    for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 2 * kEpiWarps * 32); }
    // readers of a unit slot: the even CTA's MMA warp and epilogue warps, the odd CTA's TMA thread and
    // epilogue warps
    for (int i = 0; i < UNIT_RING; ++i) { mbar_init(&u_full[i], 1); mbar_init(&u_empty[i], 2 + 2 * kEpiWarps); }
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_holder, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int u_next = pair, drawn = -1;
      for (int ku = 0; ok; ++ku) {
        int u = pair + ku * npairs;
        if (args.sched) {
          if (leader) {
            u = u_next;
            if (ku > 0 && !unit_put_pair(u_full, u_empty, u_slot, ku - 1, u)) break;
            if (u < args.units) drawn = u_next = unit_draw(args, npairs);
          } else if (ku > 0) {
            u = unit_get_pair(u_full, u_empty, u_slot, ku - 1, false);
            if (u < 0) break;
          }
        }
        if (u >= args.units) break;
        const int tile = u / args.splits, split = u % args.splits;
        const int m0 = (tile / args.n_tiles_n) * (2 * BM) + (int)rank * BM;  // this CTA's rows
        const int n0 = (tile % args.n_tiles_n) * BN + (int)rank * (BN / 2);  // this CTA's half of B
        const int kb0 = split * args.kb_per_split;
        const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!bounded_wait(&empty[stage], phase ^ 1u, DEV_TIMEOUT_EMPTY)) { ok = false; break; }
          uint8_t* sA = smem + stage * L::STAGE_BYTES;
          uint8_t* sB = sA + L::A_BYTES;
          const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);  // the even CTA's barrier
          if (leader) mbar_arrive_expect_tx(&full[stage], 2 * L::STAGE_BYTES);
          const int k0 = kb * BK;
          if (!A_MN) {
            tma_load_2d_pair(sA, &tmA, bar, k0, m0);
          } else {
#pragma unroll
            for (int c = 0; c < BM / ATOM; ++c) tma_load_2d_pair(sA + c * BK * 128, &tmA, bar, m0 + c * ATOM, k0);
          }
          if (!B_MN) {
            tma_load_2d_pair(sB, &tmB, bar, k0, n0);
          } else {
#pragma unroll
            for (int c = 0; c < (BN / 2) / ATOM; ++c)
              tma_load_2d_pair(sB + c * BK * 128, &tmB, bar, n0 + c * ATOM, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
      }
      if (leader) unit_settle(args, drawn, npairs);
    }
  } else if (warp == 1) {
    // ------------------------------------------------ MMA issuer (even CTA only)
    if (leader) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int ku = 0; ok; ++ku) {
        const int u = (ku == 0 || !args.sched) ? pair + ku * npairs
                                               : unit_get_pair(u_full, u_empty, u_slot, ku - 1, true);
        if (u < 0 || u >= args.units) break;
        const int split = u % args.splits;
        const int kb0 = split * args.kb_per_split;
        const int kb1 = min(args.k_blocks, kb0 + args.kb_per_split);
        // both CTAs' epilogues have drained accumulator `acc`
        if (!__all_sync(0xffffffffu, bounded_wait_cluster(&acc_empty[acc], acc_phase ^ 1u, DEV_TIMEOUT_ACC))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!bounded_wait_warp(&full[stage], phase, DEV_TIMEOUT_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_base = smem_u32(smem + stage * L::STAGE_BYTES);
          const uint32_t b_base = a_base + L::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / UMMA_K; ++k) {
            uint64_t ad, bd;
            if (!A_MN) ad = smem_desc_sw128(a_base + k * UMMA_K * 2, 16, 1024);
            else       ad = smem_desc_sw128(a_base + k * UMMA_K * 128, BK * 128, 1024);
            if (!B_MN) bd = smem_desc_sw128(b_base + k * UMMA_K * 2, 16, 1024);
            else       bd = smem_desc_sw128(b_base + k * UMMA_K * 128, BK * 128, 1024);
            umma_f16_pair_w(d_tmem, ad, bd, IDESC, (kb > kb0 || k > 0) ? 1u : 0u);
          }
          umma_commit_pair_w(&empty[stage], 0x3);
          if (++stage == STAGES) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair_w(&acc_full[acc], 0x3);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
    }
  } else {
    // ------------------------------------------------ epilogue (both CTAs, own TMEM half)
    const int ew = warp - 2;
    const int quarter = warp & 3;
    const int col_half = ew >> 2;
    const uint32_t stg = smem_u32(smem + L::EPI_OFF + ew * kStgBytes);
    const bool fast_ok = ((args.flags & ZL_EPI_OUT_F32) ? (args.N % 4 == 0) : (args.N % 8 == 0)) &&
                         (!(args.flags & ZL_EPI_ROPE) || args.epi.head_dim % 32 == 0);
    const bool use_tma = fast_ok && args.tma_out;
    const uint32_t acc_empty_leader[2] = {mapa_shared(smem_u32(&acc_empty[0]), 0),
                                          mapa_shared(smem_u32(&acc_empty[1]), 0)};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int ku = 0;; ++ku) {
      const int u = (ku == 0 || !args.sched) ? pair + ku * npairs
                                             : unit_get_pair(u_full, u_empty, u_slot, ku - 1, true);
      if (u < 0 || u >= args.units) break;
      const int tile = u / args.splits, split = u % args.splits;
      const int m0 = (tile / args.n_tiles_n) * (2 * BM) + (int)rank * BM;
      const int n0 = (tile % args.n_tiles_n) * BN;
      if constexpr (KIND >= 0) epi_prefetch_l2<BN, KIND>(args, m0 + quarter * 32 + lane, n0 + col_half * (BN / 2));
      if (!bounded_wait_warp(&acc_full[acc], acc_phase, DEV_TIMEOUT_ACC)) break;
      tc_fence_after();
      const int r0 = m0 + quarter * 32;
      const uint32_t t_row = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      if constexpr (KIND >= 0) {  // bf16 output by TMA store, pipelined (the host chose KIND)
        if (r0 < args.M) drain_bf16_tma<BN, KIND>(args, &tmD, t_row, stg, lane, r0, n0, col_half * (BN / 2));
      } else
#pragma unroll 1
      for (int c = col_half * (BN / 2); c < (col_half + 1) * (BN / 2); c += 32) {
        uint32_t raw[32];
        tmem_ld32(t_row + (uint32_t)c, raw);
        tmem_ld_wait();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
        const int c0 = n0 + c;
        if (c0 >= args.N || r0 >= args.M) continue;
        const bool full_chunk = fast_ok && (c0 + 32 <= args.N);
        if (use_tma) stg_reclaim(lane);
        if (args.split_direct) {
          // every split adds its partial into D; the adds of different splits land in any order
          chunk_tma_out(&tmD, stg, lane, r0, c0, v, true, true);
        } else if (args.splits > 1) {
          // a box must not run past row M: the workspace map would carry it into the next split
          if (full_chunk) partial_chunk(args, stg, lane, split, r0, c0, v, (use_tma && r0 + 32 <= args.M) ? &tmW : nullptr);
          else if (r0 + lane < args.M) {
            float* out = args.ws + ((size_t)split * args.M + r0 + lane) * args.N + c0;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (c0 + j < args.N) out[j] = v[j];
          }
        } else if (full_chunk) {
          epilogue_chunk(args, stg, lane, r0, c0, v, use_tma ? &tmD : nullptr);
        } else {
          epilogue_store32(args, r0 + lane, c0, v);
        }
      }
      tc_fence_before();
      mbar_arrive_cluster(acc_empty_leader[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
    if (use_tma && lane == 0) bulk_wait0();  // this warp's output copies are complete
  }

  // The even CTA's MMAs read both CTAs' shared memory and write both TMEMs: neither CTA may
  // leave (or free its TMEM) before both are done.
  tc_fence_before();
  __syncwarp();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// Sums split-K partials and applies the epilogue: one thread per 32 columns of a row.
__global__ void splitk_reduce_kernel(const GemmArgs args) {
  const int chunks = (args.N + 31) / 32;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)args.M * chunks) return;
  const int r = (int)(idx / chunks), c0 = (int)(idx % chunks) * 32;
  const int nvalid = min(32, args.N - c0);
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = 0.f;
  for (int s = 0; s < args.splits; ++s) {
    const float* p = args.ws + ((size_t)s * args.M + r) * args.N + c0;
    if (nvalid == 32 && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4 w = __ldg(reinterpret_cast<const float4*>(p) + q);
        v[q * 4] += w.x; v[q * 4 + 1] += w.y; v[q * 4 + 2] += w.z; v[q * 4 + 3] += w.w;
      }
    } else {
      for (int j = 0; j < nvalid; ++j) v[j] += p[j];
    }
  }
  epilogue_store32(args, r, c0, v);
}

// Split-K sum for plain fp32 outputs (no epilogue beyond OUT_F32 / ACCUM), N % 4 == 0: one
// thread per 4 columns of a row, the splits summed with four loads in flight.
__global__ void splitk_reduce_f32_kernel(const float* __restrict__ ws, float* __restrict__ out, int M, int N, int splits,
                                         int accum) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t n4 = (int64_t)M * N / 4;
  if (idx >= n4) return;
  const float4* p = reinterpret_cast<const float4*>(ws) + idx;
  const int64_t sstride = (int64_t)M * N / 4;
  float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0, a2 = a0, a3 = a0;
  int s = 0;
  for (; s + 3 < splits; s += 4) {
    const float4 u0 = __ldg(p + s * sstride), u1 = __ldg(p + (s + 1) * sstride), u2 = __ldg(p + (s + 2) * sstride),
                 u3 = __ldg(p + (s + 3) * sstride);
    a0.x += u0.x; a0.y += u0.y; a0.z += u0.z; a0.w += u0.w;
    a1.x += u1.x; a1.y += u1.y; a1.z += u1.z; a1.w += u1.w;
    a2.x += u2.x; a2.y += u2.y; a2.z += u2.z; a2.w += u2.w;
    a3.x += u3.x; a3.y += u3.y; a3.z += u3.z; a3.w += u3.w;
  }
  for (; s < splits; ++s) {
    const float4 u = __ldg(p + s * sstride);
    a0.x += u.x; a0.y += u.y; a0.z += u.z; a0.w += u.w;
  }
  float4 r = make_float4((a0.x + a1.x) + (a2.x + a3.x), (a0.y + a1.y) + (a2.y + a3.y),
                         (a0.z + a1.z) + (a2.z + a3.z), (a0.w + a1.w) + (a2.w + a3.w));
  float4* o = reinterpret_cast<float4*>(out) + idx;
  if (accum) {
    const float4 prev = *o;
    r.x += prev.x; r.y += prev.y; r.z += prev.z; r.w += prev.w;
  }
  *o = r;
}

// SIMT fallback for fp32 shapes whose rows are not 16-byte aligned (tiny
// test shapes, odd K): 64x64 tile, 4x4 outputs per thread, k ascending.
template <bool A_MN, bool B_MN>
__global__ void gemm_simt_f32_kernel(const float* __restrict__ A, const float* __restrict__ B, float* __restrict__ D,
                                     int M, int N, int K, int flags, zl_epilogue epi) {
  __shared__ float As[16][64 + 1];
  __shared__ float Bs[16][64 + 1];
  const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
  const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < K; k0 += 16) {
    for (int i = threadIdx.x; i < 16 * 64; i += 256) {
      const int kk = i / 64, mm = i % 64;
      const int gm = m0 + mm, gk = k0 + kk;
      float a = 0.f, b = 0.f;
      if (gm < M && gk < K) a = A_MN ? A[(size_t)gk * M + gm] : A[(size_t)gm * K + gk];
      const int gn = n0 + mm;
      if (gn < N && gk < K) b = B_MN ? B[(size_t)gk * N + gn] : B[(size_t)gn * K + gk];
      As[kk][mm] = a;
      Bs[kk][mm] = b;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk)
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(As[kk][ty * 4 + i], Bs[kk][tx * 4 + j], acc[i][j]);
    __syncthreads();
  }
  for (int i = 0; i < 4; ++i)
    for (int j = 0; j < 4; ++j) {
      const int r = m0 + ty * 4 + i, c = n0 + tx * 4 + j;
      if (r < M && c < N) {
        float v = acc[i][j];
        if (flags & ZL_EPI_BIAS) v += epi.bias[c];
        if (flags & ZL_EPI_RELU) v = fmaxf(v, 0.f);
        float* out = D + (size_t)r * N + c;
        *out = (flags & ZL_EPI_ACCUM) ? *out + v : v;
      }
    }
}

// ------------------------------------------------------------------ host side
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int sm_count() {
  static int count[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (count[dev] == 0) {
    int c = 0;
    cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
    count[dev] = c > 0 ? c : 148;
  }
  return count[dev];
}

// 2-D tiled map over a row-major [rows, inner] matrix with a box of [box_rows, box_inner].
// A 2-D map over `rows` rows of `inner` elements; consecutive rows are `row_stride` elements apart
// (0: packed rows), so a map can cover a column range of a wider matrix.
bool make_map(CUtensorMap* map, const void* ptr, bool is_f32, uint64_t inner, uint64_t rows, uint32_t box_inner,
              uint32_t box_rows, CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B, uint64_t row_stride = 0) {
  EncodeTiledFn enc = get_encode();
  if (!enc) return false;
  const uint64_t esz = is_f32 ? 4 : 2;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {(row_stride ? row_stride : inner) * esz};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, is_f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2,
                   const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct Plan {
  int bn, splits, n_tiles_n, tiles, k_blocks, kb_per_split, units;
};

Plan make_plan(int M, int N, int K, int BK, bool out_allows_split) {
  Plan p;
  p.bn = (N <= 128) ? 128 : 256;
  p.n_tiles_n = (N + p.bn - 1) / p.bn;
  p.tiles = ((M + BM - 1) / BM) * p.n_tiles_n;
  p.k_blocks = (K + BK - 1) / BK;
  const int sms = sm_count();
  int best = 1;
  if (out_allows_split && p.tiles < sms && p.k_blocks >= 8) {
    double best_t = 1e30;
    const int smax = std::min(16, p.k_blocks / 4);
    for (int s = 1; s <= smax; ++s) {
      const int units = p.tiles * s;
      const int waves = (units + sms - 1) / sms;
      const double t = (double)waves * ((p.k_blocks + s - 1) / s) + 0.5 * s;  // reduce cost grows with s
      if (t < best_t) { best_t = t; best = s; }
    }
  }
  p.kb_per_split = (p.k_blocks + best - 1) / best;
  p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  p.units = p.tiles * p.splits;
  return p;
}

template <typename T, int BN, int STAGES, bool A_MN, bool B_MN, int KIND>
cudaError_t launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& mw,
                      const GemmArgs& a, int grid, cudaStream_t st) {
  using E = Elem<T>;
  using L = Smem<BN, STAGES, E::bytes>;
  auto kern = gemm_tc_kernel<T, BN, STAGES, A_MN, B_MN, KIND>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, L::TOTAL, st>>>(ma, mb, md, mw, a);
  return cudaGetLastError();
}

// Kernel instances: the pipelined bf16 epilogue kinds exist for A K-major products (forward and
// dX), whose outputs are bf16; dW products (A MN-major) write fp32 through the general path.
template <typename T, int BN, int STAGES, bool B_MN>
cudaError_t launch_kind(int kind, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md,
                        const CUtensorMap& mw, const GemmArgs& a, int grid, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    switch (kind) {
      case EK_PLAIN: return launch_tc<T, BN, STAGES, false, B_MN, EK_PLAIN>(ma, mb, md, mw, a, grid, st);
      case EK_RESIDUAL: return launch_tc<T, BN, STAGES, false, B_MN, EK_RESIDUAL>(ma, mb, md, mw, a, grid, st);
      case EK_MASK: return launch_tc<T, BN, STAGES, false, B_MN, EK_MASK>(ma, mb, md, mw, a, grid, st);
      case EK_ROPE: return launch_tc<T, BN, STAGES, false, B_MN, EK_ROPE>(ma, mb, md, mw, a, grid, st);
      case EK_MASKBITS: return launch_tc<T, BN, STAGES, false, B_MN, EK_MASKBITS>(ma, mb, md, mw, a, grid, st);
      default: break;
    }
  }
  return launch_tc<T, BN, STAGES, false, B_MN, -1>(ma, mb, md, mw, a, grid, st);
}

template <typename T, int BN, int STAGES>
cudaError_t dispatch_major(bool a_mn, bool b_mn, int kind, const CUtensorMap& ma, const CUtensorMap& mb,
                           const CUtensorMap& md, const CUtensorMap& mw, const GemmArgs& a, int grid, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_kind<T, BN, STAGES, false>(kind, ma, mb, md, mw, a, grid, st);
  if (!a_mn && b_mn) return launch_kind<T, BN, STAGES, true>(kind, ma, mb, md, mw, a, grid, st);
  if (a_mn && !b_mn) return launch_tc<T, BN, STAGES, true, false, -1>(ma, mb, md, mw, a, grid, st);
  return launch_tc<T, BN, STAGES, true, true, -1>(ma, mb, md, mw, a, grid, st);
}

// Two-SM variant: tiles of 256 rows (a CTA pair), grid = 2 x pairs, cluster of 2.
Plan make_plan_pair(int M, int N, int K) {
  Plan p;
  p.bn = (N <= 128) ? 128 : 256;
  p.n_tiles_n = (N + p.bn - 1) / p.bn;
  p.tiles = ((M + 2 * BM - 1) / (2 * BM)) * p.n_tiles_n;
  p.k_blocks = (K + 63) / 64;
  const int pairs = sm_count() / 2;
  int best = 1;
  if (p.tiles < pairs && p.k_blocks >= 8) {
    // Cost in k-block times of one pair tile (~0.3 us): each round of units costs its k-blocks plus
    // a fixed ~16 (pipeline fill, accumulator drain), and each split adds its fp32 partial of the
    // whole output to D (M*N*4 bytes through L2, ~1.5 MB per k-block time).  Measured on the weight
    // gradients of the 26M model (K = 32768) this picks the fastest split count of a sweep of
    // 1..16 for every shape (output head 152.6 us at 4 splits against 170.0 us at the 16 the
    // earlier waves-only model chose; FF2 59.4 against 68.6 us).
    double best_t = 1e30;
    const int smax = std::min(16, p.k_blocks / 4);
    const double red = (double)M * N * 4.0 / 1.5e6;
    for (int s = 1; s <= smax; ++s) {
      const int units = p.tiles * s;
      const int rounds = (units + pairs - 1) / pairs;
      const double t = (double)rounds * ((p.k_blocks + s - 1) / s + 16) + red * s;
      if (t < best_t) { best_t = t; best = s; }
    }
  }
  p.kb_per_split = (p.k_blocks + best - 1) / best;
  p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;
  p.units = p.tiles * p.splits;
  return p;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int KIND>
cudaError_t launch_tc2(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md, const CUtensorMap& mw,
                       const GemmArgs& a, int pairs, cudaStream_t st) {
  using L = Smem2<BN, STAGES>;
  auto kern = gemm_tc2_kernel<BN, STAGES, A_MN, B_MN, KIND>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::TOTAL;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // persistent pairs: no more than can be resident at once (one CTA per SM)
  static int max_clusters[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64) {
    if (max_clusters[dev] == 0) {
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = pairs;
      }
      max_clusters[dev] = n;
    }
    if (pairs > max_clusters[dev]) cfg.gridDim = dim3(2 * max_clusters[dev], 1, 1);
  }
  return cudaLaunchKernelEx(&cfg, kern, ma, mb, md, mw, a);
}

template <int BN, int STAGES, bool B_MN>
cudaError_t launch_kind2(int kind, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& md,
                         const CUtensorMap& mw, const GemmArgs& a, int pairs, cudaStream_t st) {
  switch (kind) {
    case EK_PLAIN: return launch_tc2<BN, STAGES, false, B_MN, EK_PLAIN>(ma, mb, md, mw, a, pairs, st);
    case EK_RESIDUAL: return launch_tc2<BN, STAGES, false, B_MN, EK_RESIDUAL>(ma, mb, md, mw, a, pairs, st);
    case EK_MASK: return launch_tc2<BN, STAGES, false, B_MN, EK_MASK>(ma, mb, md, mw, a, pairs, st);
    case EK_ROPE: return launch_tc2<BN, STAGES, false, B_MN, EK_ROPE>(ma, mb, md, mw, a, pairs, st);
    case EK_MASKBITS: return launch_tc2<BN, STAGES, false, B_MN, EK_MASKBITS>(ma, mb, md, mw, a, pairs, st);
    default: return launch_tc2<BN, STAGES, false, B_MN, -1>(ma, mb, md, mw, a, pairs, st);
  }
}

template <int BN, int STAGES>
cudaError_t dispatch_pair(bool a_mn, bool b_mn, int kind, const CUtensorMap& ma, const CUtensorMap& mb,
                          const CUtensorMap& md, const CUtensorMap& mw, const GemmArgs& a, int pairs, cudaStream_t st) {
  if (!a_mn && !b_mn) return launch_kind2<BN, STAGES, false>(kind, ma, mb, md, mw, a, pairs, st);
  if (!a_mn && b_mn) return launch_kind2<BN, STAGES, true>(kind, ma, mb, md, mw, a, pairs, st);
  if (a_mn && !b_mn) return launch_tc2<BN, STAGES, true, false, -1>(ma, mb, md, mw, a, pairs, st);
  return launch_tc2<BN, STAGES, true, true, -1>(ma, mb, md, mw, a, pairs, st);
}

// Which bf16 GEMMs run on the CTA-pair kernel.  Measured on B200: the pair wins once the reduction
// is long (K >= 1536: +3 to +10 %, long-K dW products and the scaled model's GEMMs reach 94-97 % of
// the measured peak) and loses a little at K = 512 with N <= 2048 (QKV, FF1 forward 53 / 65 us
// against 57 / 72 us), where the per-tile work is short; at K = 512 with a wide output (the output
// head, N = 6400) it wins again (170 against 190 us).
// ZL_GEMM_PAIR=0 / =1 forces the one-SM / pair kernel (read on every call).
bool use_pair(int M, int N, int K) {
  if (M < 2 * BM) return false;
  const char* e = getenv("ZL_GEMM_PAIR");
  if (e && e[0] == '0') return false;
  if (e && e[0] == '1') return true;
  return K >= 1024 || N >= 4096;
}
}  // namespace

bool make_tma_map(CUtensorMap* map, const void* ptr, bool is_f32, uint64_t inner, uint64_t rows, uint32_t box_inner,
                  uint32_t box_rows, int swizzle_bytes, uint64_t row_stride) {
  return make_map(map, ptr, is_f32, inner, rows, box_inner, box_rows,
                  swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B, row_stride);
}
int sm_count_current() { return sm_count(); }

int64_t gemm_workspace_floats(int M, int N, int K, int layout, int flags, bool f32_inputs) {
  (void)layout;
  (void)flags;
  const int BK = f32_inputs ? Elem<float>::BK : Elem<__nv_bfloat16>::BK;
  Plan p = make_plan(M, N, K, BK, true);
  int64_t w = p.splits > 1 ? (int64_t)p.splits * M * N : 0;
  if (!f32_inputs && M >= 2 * BM) {  // the two-SM plan may split differently
    Plan q = make_plan_pair(M, N, K);
    if (q.splits > 1) w = std::max(w, (int64_t)q.splits * M * N);
  }
  return w;
}

// Generic tcgen05 GEMM launcher (T = __nv_bfloat16 or float/tf32).
zl_status colsum_bf16_add(const zl_bf16* dy, float* db, int64_t M, int N, cudaStream_t s);

// colsum (bf16 outputs only; may be null): the column sums of the stored output are added into it,
// by the pipelined epilogue when it takes the product, else by a separate column-sum pass.
// bits_out / bits_in (bf16 outputs only, N a multiple of 32; may be null): ReLU masks as bits, written by
// this product's epilogue / read in place of epi->aux by a ZL_EPI_RELU_MASK product.
template <typename T>
zl_status gemm_tc(const T* A, const T* B, void* D, int M, int N, int K, int layout, int flags,
                  const zl_epilogue* epi, float* ws, cudaStream_t st, float* colsum = nullptr,
                  uint32_t* bits_out = nullptr, const uint32_t* bits_in = nullptr, int* sched = nullptr) {
  using E = Elem<T>;
  if (M <= 0 || N <= 0 || K <= 0) return set_error(ZL_EINVAL, "gemm: sizes must be positive (M=%d N=%d K=%d)", M, N, K);
  if (!A || !B || !D) return set_error(ZL_EINVAL, "gemm: null operand");
  if (colsum && (sizeof(T) == 4 || (flags & ZL_EPI_OUT_F32)))
    return set_error(ZL_EINVAL, "gemm: column sums are for bf16 outputs");
  const bool a_mn = !(layout & ZL_A_KMAJOR), b_mn = !(layout & ZL_B_KMAJOR);
  const bool is_f32 = sizeof(T) == 4;
  if ((flags & ZL_EPI_BIAS) && (!epi || !epi->bias)) return set_error(ZL_EINVAL, "gemm: bias flag without bias");
  if ((flags & ZL_EPI_RESIDUAL) && (!epi || !epi->residual)) return set_error(ZL_EINVAL, "gemm: residual flag without residual");
  if ((flags & ZL_EPI_RELU_MASK) && (!epi || !epi->aux) && !bits_in)
    return set_error(ZL_EINVAL, "gemm: relu-mask flag without aux");
  if ((bits_out || bits_in) && (sizeof(T) == 4 || (flags & ZL_EPI_OUT_F32) || N % 32 != 0))
    return set_error(ZL_EINVAL, "gemm: ReLU mask bits are for bf16 outputs with N a multiple of 32");
  // the epilogue writes a warp's four mask words of a row as one 16-byte store
  if (bits_out && (N % 128 != 0 || (reinterpret_cast<uintptr_t>(bits_out) & 15)))
    return set_error(ZL_EINVAL, "gemm: mask bits out need N a multiple of 128 and a 16-byte aligned buffer");
  if (bits_in && !(flags & ZL_EPI_RELU_MASK)) return set_error(ZL_EINVAL, "gemm: mask bits without the relu-mask flag");
  if ((flags & ZL_EPI_ROPE) && (!epi || !epi->rope_cos || !epi->rope_sin || epi->head_dim <= 0 || epi->rope_seq <= 0 ||
                                (epi->head_dim & 1)))
    return set_error(ZL_EINVAL, "gemm: rope flag without tables");
  // TMA needs 16-byte aligned base and row pitch.
  const int align_elems = 16 / E::bytes;
  const int a_inner = a_mn ? M : K, b_inner = b_mn ? N : K;
  if ((a_inner % align_elems) || (b_inner % align_elems) || (reinterpret_cast<uintptr_t>(A) & 15) ||
      (reinterpret_cast<uintptr_t>(B) & 15))
    return ZL_EUNSUPPORTED;
  GemmArgs a;
  a.colsum = nullptr;
  a.bits_out = nullptr;
  a.bits_in = bits_in;
  a.sched = sched;
  a.M = M; a.N = N; a.K = K;
  a.D = D; a.flags = flags;
  if (epi) a.epi = *epi; else memset(&a.epi, 0, sizeof(a.epi));
  // bf16 products of at least one 256-row tile go to the CTA-pair kernel
  const bool pair = !is_f32 && sm_count() >= 2 && use_pair(M, N, K);
  Plan p = pair ? make_plan_pair(M, N, K) : make_plan(M, N, K, E::BK, true);
  const bool direct_ok = (is_f32 || (flags & ZL_EPI_OUT_F32)) && flags == (ZL_EPI_OUT_F32 | ZL_EPI_ACCUM) &&
                         N % 32 == 0 && (reinterpret_cast<uintptr_t>(D) & 15) == 0;
  if (p.splits > 1 && ((!ws && !direct_ok) || bits_out || bits_in)) {
    // no workspace supplied, or ReLU mask bits (which only the unsplit pipelined epilogue handles):
    // a single split
    p.splits = 1; p.kb_per_split = p.k_blocks; p.units = p.tiles;
  }
  a.n_tiles_n = p.n_tiles_n; a.tiles = p.tiles; a.k_blocks = p.k_blocks; a.splits = p.splits;
  a.kb_per_split = p.kb_per_split; a.units = p.units; a.ws = ws;
  constexpr int ATOM = 128 / E::bytes;
  CUtensorMap ma, mb;
  bool ok = a_mn ? make_map(&ma, A, is_f32, M, K, ATOM, E::BK) : make_map(&ma, A, is_f32, K, M, E::BK, BM);
  const int b_box_rows = pair ? p.bn / 2 : p.bn;  // a CTA of a pair loads half of B's columns
  ok = ok && (b_mn ? make_map(&mb, B, is_f32, N, K, ATOM, E::BK) : make_map(&mb, B, is_f32, K, N, E::BK, b_box_rows));
  if (!ok) return set_error(ZL_ECUDA, "gemm: cuTensorMapEncodeTiled failed (M=%d N=%d K=%d)", M, N, K);
  // Output tensor maps for the TMA-store epilogue: D ([M, N], bf16 with 64-byte or fp32 with
  // 128-byte swizzle, 32 x 32 boxes) and the split-K workspace ([splits * M, N] fp32).  They need
  // 16-byte aligned bases and row pitches; otherwise the epilogue stores from registers.
  const bool out_f32 = is_f32 || (flags & ZL_EPI_OUT_F32);
  CUtensorMap md = ma, mw = ma;
  a.tma_out = 0;
  a.split_direct = 0;
  // An accumulating fp32 output with nothing else in the epilogue takes the splits' partials
  // directly (TMA reduce-add into D): no workspace pass and no reduction launch.
  const bool direct = p.splits > 1 && out_f32 && flags == (ZL_EPI_OUT_F32 | ZL_EPI_ACCUM) && N % 32 == 0;
  if (((reinterpret_cast<uintptr_t>(D) & 15) == 0) && (out_f32 ? N % 4 == 0 : N % 8 == 0) &&
      (p.splits == 1 || direct || (ws && (reinterpret_cast<uintptr_t>(ws) & 15) == 0))) {
    bool mok = make_map(&md, D, out_f32, N, M, 32, 32,
                        out_f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
    if (mok && p.splits > 1 && !direct) mok = make_map(&mw, ws, true, N, (uint64_t)p.splits * M, 32, 32);
    a.tma_out = mok ? 1 : 0;
    a.split_direct = (mok && direct) ? 1 : 0;
  }
  // the pipelined bf16 epilogue kind (or -1): TMA output, whole 32-column chunks, and for RoPE whole
  // 32-column head slices and 16-byte aligned tables
  int kind = -1;
  if (!is_f32 && !a_mn && a.tma_out) {
    kind = bf16_epi_kind(flags, N, p.splits);
    if (kind == EK_ROPE && (a.epi.head_dim % 32 != 0 || a.epi.rope_cols % 32 != 0 ||
                            (!a.epi.rope_pair_major &&
                             ((reinterpret_cast<uintptr_t>(a.epi.rope_cos) | reinterpret_cast<uintptr_t>(a.epi.rope_sin)) & 15))))
      kind = -1;
  }
  if (colsum && kind >= 0) a.colsum = colsum;
  if (bits_in || bits_out) {
    // the mask bits exist only in the pipelined bf16 epilogue
    if (kind < 0) return set_error(ZL_EUNSUPPORTED, "gemm: ReLU mask bits need the pipelined bf16 epilogue "
                                                    "(A K-major, 16-byte aligned output, no split-K)");
    if (bits_in) {
      if (kind != EK_MASK) return set_error(ZL_EUNSUPPORTED, "gemm: mask bits with another row-wise input");
      kind = EK_MASKBITS;
    }
    a.bits_out = bits_out;
  }
  cudaError_t e;
  if (pair) {
    const int pairs = std::min(p.units, sm_count() / 2);
    if (p.bn == 128) e = dispatch_pair<128, 8>(a_mn, b_mn, kind, ma, mb, md, mw, a, pairs, st);
    else e = dispatch_pair<256, 6>(a_mn, b_mn, kind, ma, mb, md, mw, a, pairs, st);
  } else {
    const int grid = std::min(p.units, sm_count());
    if (p.bn == 128) e = dispatch_major<T, 128, 6>(a_mn, b_mn, kind, ma, mb, md, mw, a, grid, st);
    else e = dispatch_major<T, 256, 4>(a_mn, b_mn, kind, ma, mb, md, mw, a, grid, st);
  }
  if (e != cudaSuccess) return set_error(ZL_ECUDA, "gemm launch: %s", cudaGetErrorString(e));
  if (p.splits > 1 && !a.split_direct) {
    const bool plain_f32 = (flags & ~(ZL_EPI_OUT_F32 | ZL_EPI_ACCUM)) == 0 && (flags & ZL_EPI_OUT_F32) && N % 4 == 0 &&
                           ((reinterpret_cast<uintptr_t>(D) | reinterpret_cast<uintptr_t>(ws)) & 15) == 0;
    zl_status r;
    if (plain_f32) {
      const int64_t n4 = (int64_t)M * N / 4;
      splitk_reduce_f32_kernel<<<(unsigned)((n4 + 255) / 256), 256, 0, st>>>(ws, static_cast<float*>(D), M, N, p.splits,
                                                                            (flags & ZL_EPI_ACCUM) ? 1 : 0);
      r = check_launch("splitk_reduce_f32");
    } else {
      const int64_t work = (int64_t)M * ((N + 31) / 32);
      splitk_reduce_kernel<<<(unsigned)((work + 255) / 256), 256, 0, st>>>(a);
      r = check_launch("splitk_reduce");
    }
    if (r != ZL_OK) return r;
  }
  // column sums the epilogue did not take (a shape outside the pipelined bf16 epilogue)
  if (colsum && !a.colsum) return colsum_bf16_add(reinterpret_cast<const zl_bf16*>(D), colsum, M, N, st);
  return ZL_OK;
}

zl_status gemm_simt_f32(const float* A, const float* B, float* D, int M, int N, int K, int layout, int flags,
                        const zl_epilogue* epi, cudaStream_t st) {
  zl_epilogue e;
  if (epi) e = *epi; else memset(&e, 0, sizeof(e));
  dim3 grid((N + 63) / 64, (M + 63) / 64);
  const bool a_mn = !(layout & ZL_A_KMAJOR), b_mn = !(layout & ZL_B_KMAJOR);
  if (!a_mn && !b_mn) gemm_simt_f32_kernel<false, false><<<grid, 256, 0, st>>>(A, B, D, M, N, K, flags, e);
  else if (!a_mn && b_mn) gemm_simt_f32_kernel<false, true><<<grid, 256, 0, st>>>(A, B, D, M, N, K, flags, e);
  else if (a_mn && !b_mn) gemm_simt_f32_kernel<true, false><<<grid, 256, 0, st>>>(A, B, D, M, N, K, flags, e);
  else gemm_simt_f32_kernel<true, true><<<grid, 256, 0, st>>>(A, B, D, M, N, K, flags, e);
  return check_launch("gemm_simt_f32");
}

// fp32 API GEMM on tcgen05 kind::tf32.  The kernel takes K-major operands (the reduction dimension
// contiguous).  An MN-major operand (B of A·B, both operands of Aᵀ·B) is first transposed into
// stream-ordered scratch memory (32 x 32 tiles through shared memory) and the K-major product runs
// on that copy.  (MN-major 32-bit operands would need the 32-byte-atom swizzle variant of the
// shared-memory layout, which the kernel does not implement; with the plain 128-byte swizzle the
// tensor core returns zeros for them.)  Without a caller workspace, the split-K partials of products
// with few output tiles go to the same scratch allocation.  Shapes the tensor-map rules exclude (K
// not a multiple of 4, so rows are not 16-byte multiples, or unaligned bases) run on the SIMT kernel.
zl_status gemm_f32(const float* A, const float* B, float* D, int M, int N, int K, int layout, int flags,
                   const zl_epilogue* epi, float* ws, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0) return set_error(ZL_EINVAL, "gemm: sizes must be positive");
  const bool a_mn = !(layout & ZL_A_KMAJOR), b_mn = !(layout & ZL_B_KMAJOR);
  if (K % 4 == 0) {
    const size_t na = a_mn ? (size_t)M * K : 0, nb = b_mn ? (size_t)N * K : 0;
    // split-K partials for products with few output tiles and a long reduction, when the caller
    // passes no workspace (the reference-style entry points have none)
    const size_t nw = ws ? 0 : (size_t)gemm_workspace_floats(M, N, K, ZL_A_KMAJOR | ZL_B_KMAJOR, flags, true);
    const size_t total = na + nb + nw;
    float* scratch = nullptr;
    if (total > 0 && cudaMallocAsync(reinterpret_cast<void**>(&scratch), total * sizeof(float), st) != cudaSuccess) {
      cudaGetLastError();  // no scratch memory: the SIMT kernel needs none
      scratch = nullptr;
    }
    if (nw > 0 && scratch) ws = scratch + na + nb;
    if (total == 0 || scratch) {
      const float* ak = A;
      const float* bk = B;
      zl_status s = ZL_OK;
      if (a_mn) {  // A is stored [K][M]: its K-major copy is [M][K]
        s = zl_transpose_f32(A, scratch, K, M, st);
        ak = scratch;
      }
      if (s == ZL_OK && b_mn) {  // B is stored [K][N]: its K-major copy is [N][K]
        s = zl_transpose_f32(B, scratch + na, K, N, st);
        bk = scratch + na;
      }
      if (s == ZL_OK)
        s = gemm_tc<float>(ak, bk, D, M, N, K, ZL_A_KMAJOR | ZL_B_KMAJOR, flags | ZL_EPI_OUT_F32, epi, ws, st);
      if (scratch) cudaFreeAsync(scratch, st);
      if (s != ZL_EUNSUPPORTED) return s;
    }
  }
  return gemm_simt_f32(A, B, D, M, N, K, layout, flags, epi, st);
}

int gemm_dev_error_read_and_clear() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, zl_dev_error, sizeof(int));
  if (v) {
    int z = 0;
    cudaMemcpyToSymbol(zl_dev_error, &z, sizeof(int));
  }
  return v;
}

template zl_status gemm_tc<__nv_bfloat16>(const __nv_bfloat16*, const __nv_bfloat16*, void*, int, int, int, int, int,
                                          const zl_epilogue*, float*, cudaStream_t, float*, uint32_t*,
                                          const uint32_t*, int*);

// zl_gemm_bf16 that also adds the column sums of its bf16 output into colsum (a bias gradient):
// in the epilogue when the product takes the pipelined bf16 epilogue, else by a column-sum pass.
// sched (an int, zero before the first launch, may be null) lets the CTAs draw their work units at
// run time; every GEMM given the same counter must run in one stream.
zl_status gemm_bf16_colsum(const zl_bf16* A, const zl_bf16* B, void* D, int M, int N, int K, int layout, int flags,
                           const zl_epilogue* epi, float* ws, float* colsum, cudaStream_t st, uint32_t* bits_out,
                           const uint32_t* bits_in, int* sched) {
  if (reinterpret_cast<uintptr_t>(sched) & 3) return set_error(ZL_EINVAL, "gemm: unit counters must be 4-byte aligned");
  zl_status s = gemm_tc<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(A),
                                       reinterpret_cast<const __nv_bfloat16*>(B), D, M, N, K, layout, flags, epi, ws,
                                       st, colsum, bits_out, bits_in, sched);
  if (s == ZL_EUNSUPPORTED)
    return set_error(ZL_EUNSUPPORTED, "gemm: operands must be 16-byte aligned with rows a multiple of 8");
  return s;
}

}  // namespace zl

// ------------------------------------------------------------------ C ABI
extern "C" zl_status zl_gemm_bf16(const zl_bf16* A, const zl_bf16* B, void* D, int M, int N, int K, int layout,
                                  int epi_flags, const zl_epilogue* epi, float* workspace, zl_stream stream) {
  zl_status s = zl::gemm_tc<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(A),
                                           reinterpret_cast<const __nv_bfloat16*>(B), D, M, N, K, layout, epi_flags,
                                           epi, workspace, static_cast<cudaStream_t>(stream));
  if (s == ZL_EUNSUPPORTED)
    return zl::set_error(ZL_EUNSUPPORTED, "zl_gemm_bf16: operands must be 16-byte aligned with rows a multiple of 8");
  return s;
}

extern "C" zl_status zl_gemm_bf16_colsum(const zl_bf16* A, const zl_bf16* B, void* D, int M, int N, int K, int layout,
                                         int epi_flags, const zl_epilogue* epi, float* workspace, float* colsum,
                                         zl_stream stream) {
  if (!colsum) return zl::set_error(ZL_EINVAL, "zl_gemm_bf16_colsum: null colsum");
  return zl::gemm_bf16_colsum(A, B, D, M, N, K, layout, epi_flags, epi, workspace, colsum,
                              static_cast<cudaStream_t>(stream), nullptr, nullptr, nullptr);
}

extern "C" zl_status zl_gemm_bf16_relu_bits(const zl_bf16* A, const zl_bf16* B, void* D, int M, int N, int K,
                                            int layout, int epi_flags, const zl_epilogue* epi, float* workspace,
                                            uint32_t* bits_out, const uint32_t* bits_in, zl_stream stream) {
  if (!bits_out && !bits_in) return zl::set_error(ZL_EINVAL, "zl_gemm_bf16_relu_bits: no mask bits given");
  return zl::gemm_bf16_colsum(A, B, D, M, N, K, layout, epi_flags, epi, workspace, nullptr,
                              static_cast<cudaStream_t>(stream), bits_out, bits_in, nullptr);
}

extern "C" zl_status zl_gemm_bf16_sched(const zl_bf16* A, const zl_bf16* B, void* D, int M, int N, int K, int layout,
                                        int epi_flags, const zl_epilogue* epi, float* workspace, int* unit_counters,
                                        zl_stream stream) {
  if (!unit_counters) return zl::set_error(ZL_EINVAL, "zl_gemm_bf16_sched: null unit counters");
  return zl::gemm_bf16_colsum(A, B, D, M, N, K, layout, epi_flags, epi, workspace, nullptr,
                              static_cast<cudaStream_t>(stream), nullptr, nullptr, unit_counters);
}

extern "C" int64_t zl_gemm_workspace_floats(int M, int N, int K, int layout, int epi_flags) {
  return zl::gemm_workspace_floats(M, N, K, layout, epi_flags, false);
}

// ------------------------------------------------------------------ fp32 reference API
namespace zl {
// linear.cu:59-69 compute_bias_grad_kernel: one thread per column, rows ascending, += into dB.
__global__ void bias_grad_f32_kernel(float* __restrict__ dB, const float* __restrict__ dY, int64_t M, int64_t N) {
  const int64_t n = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  float g = 0.f;
  for (int64_t i = 0; i < M; ++i) g += dY[i * N + n];
  dB[n] += g;
}
}  // namespace zl

namespace zl {
// y[m, n] += bias[n] on bf16 rows, eight columns per thread (16-byte accesses); N % 8 == 0.
__global__ void bias_add_bf16_kernel(__nv_bfloat16* __restrict__ y, const __nv_bfloat16* __restrict__ bias, int64_t M,
                                     int N) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int cpr = N / 8;
  if (idx >= M * cpr) return;
  const int n0 = (int)(idx % cpr) * 8;
  uint4* yp = reinterpret_cast<uint4*>(y) + idx;
  uint4 u = *yp;
  const uint4 bb = __ldg(reinterpret_cast<const uint4*>(bias + n0));
  uint32_t* uw = reinterpret_cast<uint32_t*>(&u);
  const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bb);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 a = unpack_bf16(uw[k]), c = unpack_bf16(bw[k]);
    uw[k] = pack_bf16(a.x + c.x, a.y + c.y);
  }
  *yp = u;
}
// db[n] += sum_m dy[m, n] (linear.cu:59-69 in bf16 storage, fp32 sums): one block per 64 columns,
// 32 row lanes x 8 column groups of 8; N % 8 == 0.
__global__ void __launch_bounds__(256) bias_grad_bf16_kernel(__nv_bfloat16* __restrict__ db,
                                                             const __nv_bfloat16* __restrict__ dy, int64_t M, int N) {
  __shared__ float red[32][65];
  const int cg = threadIdx.x & 7, rl = threadIdx.x >> 3;
  const int n0 = blockIdx.x * 64 + cg * 8;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (n0 < N) {
    for (int64_t r = rl; r < M; r += 32) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(dy + r * N + n0));
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16(w[k]);
        acc[2 * k] += f.x;
        acc[2 * k + 1] += f.y;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) red[rl][cg * 8 + j] = acc[j];
  __syncthreads();
  if (threadIdx.x < 64) {
    const int n = blockIdx.x * 64 + threadIdx.x;
    if (n < N) {
      float t = 0.f;
      for (int i = 0; i < 32; ++i) t += red[i][threadIdx.x];
      db[n] = __float2bfloat16_rn(__bfloat162float(db[n]) + t);
    }
  }
}
}  // namespace zl

// linear.cuh:21-30 in bf16 (the reference instantiates float only): Y = X W^T on the tcgen05 GEMM
// with no split-K workspace, then Y += b.  K and N multiples of 8, 16-byte aligned rows.
extern "C" zl_status zl_linear_forward_bf16(const zl_bf16* input, const zl_bf16* weight, const zl_bf16* bias,
                                            zl_bf16* output, int64_t M, int64_t K, int64_t N, int use_bias,
                                            zl_stream s) {
  if (M <= 0 || K <= 0 || N <= 0) return zl::set_error(ZL_EINVAL, "linear bf16: sizes must be positive");
  if (K % 8 || N % 8 || M >= (int64_t)1 << 31)
    return zl::set_error(ZL_EUNSUPPORTED, "linear bf16: K and N must be multiples of 8");
  cudaStream_t st = static_cast<cudaStream_t>(s);
  zl_status r = zl::gemm_tc<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(input),
                                           reinterpret_cast<const __nv_bfloat16*>(weight), output, (int)M, (int)N,
                                           (int)K, ZL_A_KMAJOR | ZL_B_KMAJOR, 0, nullptr, nullptr, st);
  if (r == ZL_EUNSUPPORTED) return zl::set_error(ZL_EUNSUPPORTED, "linear bf16: operands must be 16-byte aligned");
  if (r != ZL_OK || !use_bias || !bias) return r;
  if (reinterpret_cast<uintptr_t>(bias) & 15) return zl::set_error(ZL_EINVAL, "linear bf16: bias must be 16-byte aligned");
  const int64_t chunks = M * (N / 8);
  zl::bias_add_bf16_kernel<<<(unsigned)((chunks + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<__nv_bfloat16*>(output), reinterpret_cast<const __nv_bfloat16*>(bias), M, (int)N);
  return zl::check_launch("add_bias_kernel");
}
// linear.cuh:48-59 in bf16: dX = dY W and dW = dY^T X overwrite, dB += column sums of dY.
extern "C" zl_status zl_linear_backward_bf16(const zl_bf16* d_output, const zl_bf16* input, const zl_bf16* weight,
                                             zl_bf16* d_input, zl_bf16* d_weight, zl_bf16* d_bias, int64_t M,
                                             int64_t K, int64_t N, int use_bias, zl_stream s) {
  if (M <= 0 || K <= 0 || N <= 0) return zl::set_error(ZL_EINVAL, "linear bf16: sizes must be positive");
  if (K % 8 || N % 8 || M % 8 || M >= (int64_t)1 << 31)
    return zl::set_error(ZL_EUNSUPPORTED, "linear bf16 backward: M, K and N must be multiples of 8");
  cudaStream_t st = static_cast<cudaStream_t>(s);
  const auto dY = reinterpret_cast<const __nv_bfloat16*>(d_output);
  zl_status r = ZL_OK;
  if (d_input)
    r = zl::gemm_tc<__nv_bfloat16>(dY, reinterpret_cast<const __nv_bfloat16*>(weight), d_input, (int)M, (int)K, (int)N,
                                   ZL_A_KMAJOR, 0, nullptr, nullptr, st);
  if (r == ZL_OK && d_weight)
    r = zl::gemm_tc<__nv_bfloat16>(dY, reinterpret_cast<const __nv_bfloat16*>(input), d_weight, (int)N, (int)K,
                                   (int)M, 0, 0, nullptr, nullptr, st);
  if (r == ZL_EUNSUPPORTED) return zl::set_error(ZL_EUNSUPPORTED, "linear bf16: operands must be 16-byte aligned");
  if (r != ZL_OK || !use_bias || !d_bias) return r;
  if (reinterpret_cast<uintptr_t>(d_output) & 15) return zl::set_error(ZL_EINVAL, "linear bf16: dY must be 16-byte aligned");
  zl::bias_grad_bf16_kernel<<<(unsigned)((N + 63) / 64), 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(d_bias), dY,
                                                                       M, (int)N);
  return zl::check_launch("compute_bias_grad_kernel");
}

// matmul.cuh:20/:68  C[M,N] = A[M,K] B[K,N]
extern "C" zl_status zl_matmul_f32(const float* A, const float* B, float* C, int M, int N, int K, zl_stream s) {
  return zl::gemm_f32(A, B, C, M, N, K, ZL_A_KMAJOR, 0, nullptr, nullptr, static_cast<cudaStream_t>(s));
}
// matmul.cuh:36/:99  C[K,N] = A[M,K]^T B[M,N]
extern "C" zl_status zl_matmul_at_b_f32(const float* A, const float* B, float* C, int M, int N, int K, zl_stream s) {
  return zl::gemm_f32(A, B, C, K, N, M, 0, 0, nullptr, nullptr, static_cast<cudaStream_t>(s));
}
// matmul.cuh:52/:83  C[M,N] = A[M,K] B[N,K]^T
extern "C" zl_status zl_matmul_a_bt_f32(const float* A, const float* B, float* C, int M, int N, int K, zl_stream s) {
  return zl::gemm_f32(A, B, C, M, N, K, ZL_A_KMAJOR | ZL_B_KMAJOR, 0, nullptr, nullptr, static_cast<cudaStream_t>(s));
}
// linear.cuh:21-30
extern "C" zl_status zl_linear_forward_f32(const float* input, const float* weight, const float* bias, float* output,
                                           int64_t M, int64_t K, int64_t N, int use_bias, zl_stream s) {
  zl_epilogue e;
  memset(&e, 0, sizeof(e));
  e.bias = bias;
  const int flags = (use_bias && bias) ? ZL_EPI_BIAS : 0;
  return zl::gemm_f32(input, weight, output, (int)M, (int)N, (int)K, ZL_A_KMAJOR | ZL_B_KMAJOR, flags, &e, nullptr,
                      static_cast<cudaStream_t>(s));
}
// linear.cuh:48-59
extern "C" zl_status zl_linear_backward_f32(const float* d_output, const float* input, const float* weight,
                                            float* d_input, float* d_weight, float* d_bias, int64_t M, int64_t K,
                                            int64_t N, int use_bias, zl_stream s) {
  cudaStream_t st = static_cast<cudaStream_t>(s);
  zl_status r = ZL_OK;
  if (d_input) r = zl::gemm_f32(d_output, weight, d_input, (int)M, (int)K, (int)N, ZL_A_KMAJOR, 0, nullptr, nullptr, st);
  if (r != ZL_OK) return r;
  if (d_weight) r = zl::gemm_f32(d_output, input, d_weight, (int)N, (int)K, (int)M, 0, 0, nullptr, nullptr, st);
  if (r != ZL_OK) return r;
  if (use_bias && d_bias) {
    zl::bias_grad_f32_kernel<<<(unsigned)((N + 255) / 256), 256, 0, st>>>(d_bias, d_output, M, N);
    r = zl::check_launch("compute_bias_grad_kernel");
  }
  return r;
}

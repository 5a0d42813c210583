// attention_tc.cu -- causal flash-attention forward on tcgen05 / TMEM (sm_100a).
//
// One CTA computes 128 query rows of one (batch, head) against key blocks of
// 128 (causal: blocks 0..q_block).  Per key block j:
//   MMA warp:      S = Q K_j^T             (M=128, N=128, K=64; A, B K-major in smem; S fp32 in TMEM)
//   softmax warps: row max / exp2 / row sum from S (two passes over TMEM), P = bf16(exp2(S - m))
//                  written back over the S columns of TMEM; O rescaled in TMEM by exp2(m_old - m_new)
//   MMA warp:      O += P V_j              (M=128, N=64, K=128; A = P from TMEM, B = V MN-major in smem)
// Q/K/V tiles arrive by TMA (128-byte swizzle) straight from the packed qkv
// activation [B*S, 3E]; K/V are double buffered.  TMEM holds two S/P buffers
// (128 columns each) and O (64 columns): the MMA warp computes S for block j+1
// while the softmax warps work on block j.  The softmax reads all 128 scores
// of its row with one TMEM round trip and uses the MUFU ex2 instruction.
// Every wait is bounded (common.cuh).  The result matches the mma.sync kernel's definition:
// probabilities rounded to bf16 before P.V, row sums from the unrounded
// values, lse = natural log-sum-exp of the scaled scores.
#include <cmath>
#include <cstdlib>

#include <initializer_list>
#include <type_traits>

#include "common.cuh"

namespace zl {
bool make_tma_map(CUtensorMap* map, const void* ptr, bool is_f32, uint64_t inner, uint64_t rows, uint32_t box_inner,
                  uint32_t box_rows, int swizzle_bytes = 128, uint64_t row_stride = 0);
int sm_count_current();

namespace fatc {

constexpr int BQ = 128, BKV = 128, D = 64;
constexpr int THREADS = 192;          // warp 0 TMA, warp 1 MMA, warps 2-5 softmax / epilogue
constexpr int TILE_BYTES = 128 * 128; // 128 rows x 64 bf16
constexpr uint32_t TMEM_COLS = 512;   // forward: S/P buffer b at [128 b, 128 b + 128), O at [256, 256 + Dh)
constexpr uint32_t O_COL = 256;
constexpr uint32_t IDESC_S = make_idesc(1, 128, 128, 0, 0);  // bf16, M=128, N=128, A/B K-major

// Forward shapes by head dim: a 128-row tile of Q, K or V is Dh/64 swizzle atoms of [128][64] bf16
// side by side (16 KB each); K / V stages fill the rest of shared memory.
template <int DH>
struct Fwd {
  static constexpr int ATOMS = DH / 64;
  static constexpr int T_BYTES = ATOMS * TILE_BYTES;
  static constexpr int KVST = DH == 64 ? 4 : 3;  // loads run KVST-1 blocks ahead
  static constexpr int SMEM_Q = 0, SMEM_K = T_BYTES, SMEM_V = SMEM_K + KVST * T_BYTES;
  static constexpr int SMEM_BAR = SMEM_V + KVST * T_BYTES;
  static constexpr int SMEM_TOTAL = SMEM_BAR + 128 + 1024;
  static constexpr uint32_t IDESC_O = make_idesc(1, 128, DH, 0, 1);  // M=128, N=Dh, A (TMEM), B MN-major
  static_assert(SMEM_TOTAL <= 227 * 1024, "shared memory");
};

enum : int { DEV_TIMEOUT_ATTN = 11 };

__device__ __forceinline__ float fast_exp2(float x) {  // MUFU ex2 (inputs <= 0 here; -inf -> 0)
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {  // sm_100 three-input maximum
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <int DH>
__global__ void __launch_bounds__(THREADS, 1)
    fa_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, __nv_bfloat16* __restrict__ out,
                     float* __restrict__ lse, int S, int H, float scale_log2) {
  using C = Fwd<DH>;
  constexpr int KVST = C::KVST, SMEM_Q = C::SMEM_Q, SMEM_K = C::SMEM_K, SMEM_V = C::SMEM_V, SMEM_BAR = C::SMEM_BAR;
  constexpr int T_BYTES = C::T_BYTES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SMEM_BAR);
  uint64_t* q_full = bar + 0;
  uint64_t* kv_full = bar + 1;              // [KVST]
  uint64_t* kv_empty = bar + 1 + KVST;      // [KVST]
  uint64_t* s_full = bar + 1 + 2 * KVST;    // [2]
  uint64_t* p_full = s_full + 2;
  uint64_t* o_full = s_full + 3;
  uint64_t* drain = s_full + 4;             // final commit: every MMA of this CTA has retired
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_full + 5);

  const int E = H * DH;
  const int nq = S / BQ;
  const int qb = nq - 1 - (int)(blockIdx.x % nq);  // heavy blocks first
  const int bh = blockIdx.x / nq, b = bh / H, h = bh % H;
  const int row0 = b * S + qb * BQ;                // first query row in the packed activation
  const int nkv = qb + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < KVST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&s_full[i], 1);
    mbar_init(p_full, 128);
    mbar_init(o_full, 1);
    mbar_init(drain, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, T_BYTES);
#pragma unroll
      for (int a = 0; a < C::ATOMS; ++a)
        tma_load_2d(smem + SMEM_Q + a * TILE_BYTES, &tm_q, q_full, h * DH + a * 64, row0);
      int issued = 0;
      for (int j = 0; j < nkv; ++j) {
        const int st = j % KVST;
        const uint32_t ph = (j / KVST) & 1;
        if (!bounded_wait(&kv_empty[st], ph ^ 1u, DEV_TIMEOUT_ATTN)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * T_BYTES);
        const int krow = b * S + j * BKV;
#pragma unroll
        for (int a = 0; a < C::ATOMS; ++a) {
          tma_load_2d(smem + SMEM_K + st * T_BYTES + a * TILE_BYTES, &tm_k, &kv_full[st], h * DH + a * 64, krow);
          tma_load_2d(smem + SMEM_V + st * T_BYTES + a * TILE_BYTES, &tm_v, &kv_full[st], h * DH + a * 64,
                      krow);
        }
        issued = j + 1;
      }
      // no copy may still be landing in shared memory when the CTA exits
      bounded_wait(q_full, 0, DEV_TIMEOUT_ATTN);
      for (int j = issued - KVST < 0 ? 0 : issued - KVST; j < issued; ++j)
        bounded_wait(&kv_full[j % KVST], (j / KVST) & 1, DEV_TIMEOUT_ATTN);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t sq = smem_u32(smem + SMEM_Q);
    auto issue_s = [&](int j) {  // S_j = Q K_j^T into TMEM buffer j & 1 (K from stage j % KVST)
      const int sb = j & 1;
      const uint32_t sk = smem_u32(smem + SMEM_K + (j % KVST) * T_BYTES);
#pragma unroll
      for (int k = 0; k < DH / 16; ++k) {  // 16 head dims per MMA: atom k / 4, 32 bytes per step inside it
        const uint32_t off = (uint32_t)((k >> 2) * TILE_BYTES + (k & 3) * 32);
        umma_f16_w(tmem + (uint32_t)(sb * BKV), smem_desc_sw128(sq + off, 16, 1024),
                 smem_desc_sw128(sk + off, 16, 1024), IDESC_S, k > 0 ? 1u : 0u);
      }
      umma_commit_w(&s_full[sb]);
    };
    bool ok = bounded_wait_warp(q_full, 0, DEV_TIMEOUT_ATTN) && bounded_wait_warp(&kv_full[0], 0, DEV_TIMEOUT_ATTN);
    if (ok) {
      tc_fence_after();
      issue_s(0);
    }
    for (int j = 0; j < nkv && ok; ++j) {
      const int sb = j & 1, st = j % KVST;
      if (j + 1 < nkv) {
        // K_{j+1} resident, and buffer (j+1)&1 free: P_{j-1} (in that buffer) consumed by P.V of block j-1
        if (!bounded_wait_warp(&kv_full[(j + 1) % KVST], ((j + 1) / KVST) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        if (j >= 1 && !bounded_wait_warp(o_full, (j - 1) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        tc_fence_after();
        issue_s(j + 1);
      }
      if (!bounded_wait_warp(p_full, j & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
      tc_fence_after();
      const uint32_t sv = smem_u32(smem + SMEM_V + st * T_BYTES);
#pragma unroll
      for (int k = 0; k < BKV / 16; ++k)  // 16 keys per MMA: P columns k*8.., V rows k*16.. (atoms TILE_BYTES apart)
        umma_f16_ts_w(tmem + O_COL, tmem + (uint32_t)(sb * BKV + k * 8),
                    smem_desc_sw128(sv + k * 16 * 128, TILE_BYTES, 1024), C::IDESC_O, (j > 0 || k > 0) ? 1u : 0u);
      umma_commit_w(o_full);
      umma_commit_w(&kv_empty[st]);
    }
    // TMEM is freed below only after every MMA issued here has retired
    umma_commit_w(drain);
    bounded_wait_warp(drain, 0, DEV_TIMEOUT_ATTN);
  } else {
    // ------------------------------------------------------------ softmax + epilogue (one row per thread)
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    const int q_pos = qb * BQ + r_local;  // position inside the sequence
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      const int st = j & 1;
      if (!bounded_wait_warp(&s_full[st], (j >> 1) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
      tc_fence_after();
      const uint32_t t_s = t_lane + (uint32_t)(st * BKV);
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(t_s + (uint32_t)(c * 32), r[c]);
      tmem_ld_wait();
      const bool diag = (j == nkv - 1);
      const int key0 = j * BKV;
      float corr = 1.f;
      bool raise = false;
      // The diagonal block (the only one with masked keys) is a separate instance, so the others
      // carry no per-element mask.
      auto block = [&](auto diag_tag) {
        constexpr bool DIAG = decltype(diag_tag)::value;
        auto val = [&](int c, int i) {
          const float v = __uint_as_float(r[c][i]);
          return (DIAG && key0 + c * 32 + i > q_pos) ? -INFINITY : v;
        };
        // row maximum of the raw scores (the scale is positive, so it commutes with max); eight
        // independent partial maxima keep the dependency chains short
        float mxp[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mxp[k] = val(0, k);
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c > 0 || i >= 8) mxp[i & 7] = fmaxf(mxp[i & 7], val(c, i));
        const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                               fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
        // Lazy rescaling: the running maximum m (log2 units) is only raised when a lane's new
        // maximum exceeds it by more than 8, so P = exp2(s - m) stays below 2^8 and O needs no
        // correction in most blocks.  The decision is per warp (TMEM access is warp-wide).
        const float m_cand = fmaxf(m, mx * scale_log2);
        raise = __any_sync(0xffffffffu, m_cand > m + 8.f);
        if (raise) {
          corr = fast_exp2(m - m_cand);  // m = -inf on the first block -> 0
          m = m_cand;
        }
        const float neg_m = -m;
        float sp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // partial row sums
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float p0 = fast_exp2(fmaf(val(c, i), scale_log2, neg_m));
            const float p1 = fast_exp2(fmaf(val(c, i + 1), scale_log2, neg_m));
            sp[i & 7] += p0;
            sp[(i + 1) & 7] += p1;
            pk[i >> 1] = pack_bf16(p0, p1);
          }
          tmem_st16(t_s + (uint32_t)(c * 16), pk);  // P over the consumed S columns
        }
        const float sum = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
        l = l * corr + sum;
      };
      if (diag) block(std::integral_constant<bool, true>{});
      else block(std::integral_constant<bool, false>{});
      if (raise && j > 0) {  // O *= corr once the previous P.V has landed
        if (!bounded_wait_warp(o_full, (j - 1) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(t_lane + O_COL + (uint32_t)(c * 32), o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
          tmem_st32(t_lane + O_COL + (uint32_t)(c * 32), o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // epilogue: O / l -> bf16, lse
    if (ok && bounded_wait_warp(o_full, (nkv - 1) & 1, DEV_TIMEOUT_ATTN)) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (size_t)(row0 + r_local) * E + h * DH;
#pragma unroll 1
      for (int c = 0; c < DH / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(t_lane + O_COL + (uint32_t)(c * 32), o);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 u;
          u.x = pack_bf16(__uint_as_float(o[q * 8 + 0]) * inv, __uint_as_float(o[q * 8 + 1]) * inv);
          u.y = pack_bf16(__uint_as_float(o[q * 8 + 2]) * inv, __uint_as_float(o[q * 8 + 3]) * inv);
          u.z = pack_bf16(__uint_as_float(o[q * 8 + 4]) * inv, __uint_as_float(o[q * 8 + 5]) * inv);
          u.w = pack_bf16(__uint_as_float(o[q * 8 + 6]) * inv, __uint_as_float(o[q * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + q * 8) = u;
        }
      }
      lse[((size_t)b * H + h) * S + qb * BQ + r_local] = (m + log2f(l)) * 0.6931471805599453f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ============================================ forward, persistent, two query tiles per work unit
// One CTA per SM walks work units (batch, head, query tiles 2p and 2p+1), heaviest first, in a
// snake order over the CTAs.  The two tiles share every K/V block load.  Each tile has its own MMA
// warp and softmax warpgroup, so two independent softmax streams run on every SM sub-partition.
// Buffers drain unit to unit: the producer loads the next unit's Q and K/V as soon as their slots
// free up, and a tile's first S of the next unit is computed while its softmax warps still write
// the previous unit's O.
//
// TMEM (512 columns): S_t at [128 t, 128 t + 128).  Head dim 64: P_t at 256 + 64 t and O_t at
// 384 + 64 t, so S of block j+1 is computed as soon as the softmax holds S_j in registers.  Head dim
// 128: O_t at 256 + 128 t, and P_t is written over the first 64 columns of S_t; S of block j+1 is
// then issued only after the P.V of block j has retired, since tcgen05 products on different
// accumulators are not ordered with respect to each other.
template <int DH>
struct FwdPP {
  static constexpr int ATOMS = DH / 64;
  static constexpr int T_BYTES = ATOMS * TILE_BYTES;
  static constexpr int KVST = DH == 64 ? 5 : 2;
  static constexpr bool SEP_P = DH == 64;
  static constexpr int SMEM_Q = 0, SMEM_K = 2 * T_BYTES, SMEM_V = SMEM_K + KVST * T_BYTES;
  static constexpr int SMEM_BAR = SMEM_V + KVST * T_BYTES;
  static constexpr int SMEM_TOTAL = SMEM_BAR + 256 + 1024;
  static constexpr uint32_t IDESC_O = make_idesc(1, 128, DH, 0, 1);  // M=128, N=Dh, A (TMEM), B MN-major
  __host__ __device__ static constexpr uint32_t s_col(int t) { return (uint32_t)(t * 128); }
  __host__ __device__ static constexpr uint32_t p_col(int t) { return SEP_P ? 256u + 64u * t : (uint32_t)(t * 128); }
  __host__ __device__ static constexpr uint32_t o_col(int t) { return SEP_P ? 384u + 64u * t : 256u + 128u * t; }
  static_assert(SMEM_TOTAL <= 227 * 1024, "shared memory");
};
constexpr int THREADS_PP = 384;  // warp 0 TMA, warps 1-2 MMA of tiles 0-1, warp 3 idle, 4-7 / 8-11 softmax

// Work unit k of a CTA (k = 0, 1, ...): snake order over the CTAs, so that a CTA that draws a heavy
// unit in one round draws a light one in the next.
__device__ __forceinline__ int pp_unit(int k, int cta, int G) { return k * G + ((k & 1) ? G - 1 - cta : cta); }

// Backward unit u -> (key block, batch-head).  Heads are taken in groups of `hg` (all of them when
// hg <= 0); inside a group the units run key-block-major, the ones with the most query blocks first.
// A group of about one wave of units keeps the rows of the fp32 dQ accumulator that are being added
// into within L2.
__device__ __forceinline__ void bwd_unit_coords(int u, int nk, int nbh, int hg, int* kb, int* bh) {
  if (hg <= 0 || hg >= nbh) {
    *kb = u / nbh;
    *bh = u % nbh;
    return;
  }
  const int grp = u / (hg * nk), r = u - grp * hg * nk;
  const int heads = min(hg, nbh - grp * hg);
  *kb = r / heads;
  *bh = grp * hg + r % heads;
}

// Backward work units are handed out at run time.  A CTA's first unit is its own index; each later
// one is the grid size plus the next value of a per-launch counter in global memory (zeroed by the
// caller's pre pass), so units still start in index order (heaviest first) but a CTA that starts
// late, because its SM is still busy with another kernel (an all-reduce on a side stream, say),
// takes fewer of them instead of holding back the end of the launch.  One thread (the TMA issuer)
// draws each unit one unit ahead, so the counter's round trip overlaps a unit's loads, and publishes
// every unit in a ring of UNIT_RING shared-memory slots; every warp of the other roles reads each
// slot once, in order, and releases it.
constexpr int UNIT_RING = 4;
struct UnitFeed {
  uint64_t* full;   // [UNIT_RING] one arrival: the drawing thread has written the slot
  uint64_t* empty;  // [UNIT_RING] one arrival per reader warp
  volatile int* slot;
  // the CTA's next unit index (>= the unit count when there are no more); one thread
  __device__ __forceinline__ int draw(int G, int* ctr) const { return G + atomicAdd(ctr, 1); }
  __device__ __forceinline__ bool put(int k, int u) const {
    const int r = k % UNIT_RING;
    if (!bounded_wait(&empty[r], ((uint32_t)(k / UNIT_RING) & 1u) ^ 1u, DEV_TIMEOUT_ATTN)) return false;
    slot[r] = u;
    mbar_arrive(&full[r]);  // release: the slot's value is visible to the thread that sees the phase
    return true;
  }
  // the CTA's k-th unit index, read by a whole warp; -1 when the wait timed out
  __device__ __forceinline__ int get(int k) const {
    const int r = k % UNIT_RING;
    if (!bounded_wait_warp(&full[r], (uint32_t)(k / UNIT_RING) & 1u, DEV_TIMEOUT_ATTN)) return -1;
    const int u = slot[r];
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&empty[r]);
    return u;
  }
};

template <int DH>
__global__ void __launch_bounds__(THREADS_PP, 1)
    fa_fwd_pp_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, __nv_bfloat16* __restrict__ out,
                     float* __restrict__ lse, int S, int H, int nunits, float scale_log2) {
  using C = FwdPP<DH>;
  constexpr int KVST = C::KVST, T_BYTES = C::T_BYTES;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + C::SMEM_BAR);
  uint64_t* q_full = bar + 0;
  uint64_t* q_empty = bar + 1;            // both tiles' last S product of the unit has retired
  uint64_t* kv_full = bar + 2;            // [KVST]
  uint64_t* kv_empty = bar + 2 + KVST;    // [KVST]: both tiles are done with the block
  uint64_t* s_full = bar + 2 + 2 * KVST;  // [2] per tile
  uint64_t* s_used = s_full + 2;          // [2] the tile's softmax warps hold S in registers
  uint64_t* p_full = s_full + 4;          // [2]
  uint64_t* pv_done = s_full + 6;         // [2]
  uint64_t* drain = s_full + 8;           // both MMA warps' last products have retired
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_full + 9);

  const int E = H * DH;
  const int npair = S / (2 * BQ);
  const int nbh = nunits / npair;
  const int G = (int)gridDim.x, cta = (int)blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // unit u: query tiles 2p, 2p+1 of (batch, head) bh; the heaviest pairs have the lowest u
  auto unit_pair = [&](int u) { return npair - 1 - u / nbh; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 2);
    for (int i = 0; i < KVST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 2);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&s_used[t], 128);
      mbar_init(&p_full[t], 128);
      mbar_init(&pv_done[t], 1);
    }
    mbar_init(drain, 2);
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t g = 0, nq_loads = 0;  // K/V blocks and Q pairs issued
      bool ok = true;
      for (int k = 0; ok; ++k) {
        const int u = pp_unit(k, cta, G);
        if (u >= nunits) break;
        const int p = unit_pair(u), bh = u % nbh, b = bh / H, h = bh % H;
        if (!bounded_wait(q_empty, (nq_loads & 1) ^ 1u, DEV_TIMEOUT_ATTN)) break;
        mbar_arrive_expect_tx(q_full, 2 * T_BYTES);
#pragma unroll
        for (int t = 0; t < 2; ++t)
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a)
            tma_load_2d(smem + C::SMEM_Q + t * T_BYTES + a * TILE_BYTES, &tm_q, q_full, h * DH + a * 64,
                        b * S + (2 * p + t) * BQ);
        ++nq_loads;
        const int nkv = 2 * p + 2;
        for (int j = 0; j < nkv; ++j) {
          const uint32_t st = g % KVST;
          if (!bounded_wait(&kv_empty[st], ((g / KVST) & 1) ^ 1u, DEV_TIMEOUT_ATTN)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[st], 2 * T_BYTES);
          const int krow = b * S + j * BKV;
#pragma unroll
          for (int a = 0; a < C::ATOMS; ++a) {
            tma_load_2d(smem + C::SMEM_K + st * T_BYTES + a * TILE_BYTES, &tm_k, &kv_full[st], h * DH + a * 64,
                        krow);
            tma_load_2d(smem + C::SMEM_V + st * T_BYTES + a * TILE_BYTES, &tm_v, &kv_full[st],
                        h * DH + a * 64, krow);
          }
          ++g;
        }
      }
      // no copy may still be landing in shared memory when the CTA exits
      if (nq_loads > 0) bounded_wait(q_full, (nq_loads - 1) & 1, DEV_TIMEOUT_ATTN);
      for (uint32_t j = g > (uint32_t)KVST ? g - KVST : 0; j < g; ++j)
        bounded_wait(&kv_full[j % KVST], (j / KVST) & 1, DEV_TIMEOUT_ATTN);
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuer of tile t
    const int t = warp - 1;
    const uint32_t sq = smem_u32(smem + C::SMEM_Q + t * T_BYTES);
    const uint32_t t_s = tmem + C::s_col(t), t_p = tmem + C::p_col(t), t_o = tmem + C::o_col(t);
    uint32_t c = 0, g = 0;  // this tile's blocks so far, K/V blocks so far
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int u = pp_unit(k, cta, G);
      if (u >= nunits) break;
      const int p = unit_pair(u);
      const int n = 2 * p + 1 + t, nkv = 2 * p + 2;
      if (!bounded_wait_warp(q_full, (uint32_t)k & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
      // S_t of block j: K/V block g + j, tile block c + j.  Its S columns must be free: read by the
      // softmax (separate P) or released by the previous P.V (P over S).
      auto issue_s = [&](int j) -> bool {
        const uint32_t use = g + (uint32_t)j, st = use % KVST;
        if (!bounded_wait_warp(&kv_full[st], (use / KVST) & 1, DEV_TIMEOUT_ATTN)) return false;
        const uint32_t prev = c + (uint32_t)j;
        if (prev > 0 && !bounded_wait_warp(C::SEP_P ? &s_used[t] : &pv_done[t], (prev - 1) & 1, DEV_TIMEOUT_ATTN))
          return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + C::SMEM_K + st * T_BYTES);
#pragma unroll
        for (int kk = 0; kk < DH / 16; ++kk) {
          const uint32_t off = (uint32_t)((kk >> 2) * TILE_BYTES + (kk & 3) * 32);
          umma_f16_w(t_s, smem_desc_sw128(sq + off, 16, 1024), smem_desc_sw128(sk + off, 16, 1024), IDESC_S,
                   kk > 0 ? 1u : 0u);
        }
        umma_commit_w(&s_full[t]);
        if (j == n - 1) umma_commit_w(q_empty);  // the tile's Q is no longer read once this retires
        return true;
      };
      ok = issue_s(0);
      for (int j = 0; j < n && ok; ++j) {
        if (C::SEP_P && j + 1 < n && !issue_s(j + 1)) { ok = false; break; }
        if (!bounded_wait_warp(&p_full[t], (c + (uint32_t)j) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = (g + (uint32_t)j) % KVST;
        const uint32_t sv = smem_u32(smem + C::SMEM_V + st * T_BYTES);
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)  // 16 keys per MMA: P columns kk*8.., V rows kk*16..
          umma_f16_ts_w(t_o, t_p + (uint32_t)(kk * 8), smem_desc_sw128(sv + kk * 16 * 128, TILE_BYTES, 1024),
                      C::IDESC_O, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit_w(&pv_done[t]);
        umma_commit_w(&kv_empty[st]);
        if (!C::SEP_P && j + 1 < n && !issue_s(j + 1)) { ok = false; break; }
      }
      if (!ok) break;
      if (t == 0) {  // tile 0 (one block fewer) releases the unit's last K/V block once it has landed
        const uint32_t use = g + (uint32_t)nkv - 1, st = use % KVST;
        if (!bounded_wait_warp(&kv_full[st], (use / KVST) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        if (lane == 0) mbar_arrive(&kv_empty[st]);
        __syncwarp();
      }
      c += (uint32_t)n;
      g += (uint32_t)nkv;
    }
    // TMEM is freed below only after every MMA issued here has retired
    umma_commit_w(drain);
    bounded_wait_warp(drain, 0, DEV_TIMEOUT_ATTN);
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax + epilogue of tile t
    const int t = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t t_s = t_lane + C::s_col(t), t_p = t_lane + C::p_col(t), t_o = t_lane + C::o_col(t);
    uint32_t c = 0;
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int u = pp_unit(k, cta, G);
      if (u >= nunits) break;
      const int p = unit_pair(u), bh = u % nbh, b = bh / H, h = bh % H;
      const int qb = 2 * p + t, n = qb + 1;
      const int q_pos = qb * BQ + r_local;
      float m = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j, ++c) {
        if (!bounded_wait_warp(&s_full[t], c & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        tc_fence_after();
        uint32_t r[4][32];
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) tmem_ld32(t_s + (uint32_t)(cc * 32), r[cc]);
        tmem_ld_wait();
        if (C::SEP_P) {  // S may now be overwritten by the next block's product
          tc_fence_before();
          mbar_arrive(&s_used[t]);
        }
        const int key0 = j * BKV;
        float corr = 1.f;
        bool raise = false;
        // The diagonal block (the only one with masked keys) is a separate instance, so the others
        // carry no per-element mask.
        auto block = [&](auto diag_tag) -> bool {
          constexpr bool DIAG = decltype(diag_tag)::value;
          auto val = [&](int cc, int i) {
            const float v = __uint_as_float(r[cc][i]);
            return (DIAG && key0 + cc * 32 + i > q_pos) ? -INFINITY : v;
          };
          float mxp[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) mxp[i] = val(0, i);
#pragma unroll
          for (int t = 0; t < 8; ++t) {  // three-input maxima: the row's 128 scores in 8 running maxima
            mxp[t] = fmax3(mxp[t], val(0, 8 + t), val(0, 16 + t));
            mxp[t] = fmaxf(mxp[t], val(0, 24 + t));
          }
#pragma unroll
          for (int cc = 1; cc < 4; ++cc)
#pragma unroll
            for (int t = 0; t < 8; ++t) {
              mxp[t] = fmax3(mxp[t], val(cc, t), val(cc, 8 + t));
              mxp[t] = fmax3(mxp[t], val(cc, 16 + t), val(cc, 24 + t));
            }
          const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                 fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
          // lazy rescaling, as in the one-tile kernel: m only rises by more than 8 (log2 units)
          const float m_cand = fmaxf(m, mx * scale_log2);
          raise = __any_sync(0xffffffffu, m_cand > m + 8.f);
          if (raise) {
            corr = fast_exp2(m - m_cand);
            m = m_cand;
          }
          // separate P columns: the previous block's P.V must have read them (and O is then current)
          if (C::SEP_P && c > 0 && !bounded_wait_warp(&pv_done[t], (c - 1) & 1, DEV_TIMEOUT_ATTN)) return false;
          const float neg_m = -m;
          float sp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float p0 = fast_exp2(fmaf(val(cc, i), scale_log2, neg_m));
              const float p1 = fast_exp2(fmaf(val(cc, i + 1), scale_log2, neg_m));
              sp[i & 7] += p0;
              sp[(i + 1) & 7] += p1;
              pk[i >> 1] = pack_bf16(p0, p1);
            }
            tmem_st16(t_p + (uint32_t)(cc * 16), pk);
          }
          const float sum = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
          l = l * corr + sum;
          return true;
        };
        const bool fine = (j == n - 1) ? block(std::integral_constant<bool, true>{})
                                       : block(std::integral_constant<bool, false>{});
        if (!fine) { ok = false; break; }
        if (raise && j > 0) {  // O *= corr once the previous P.V has landed
          if (!C::SEP_P && !bounded_wait_warp(&pv_done[t], (c - 1) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < DH / 32; ++cc) {
            uint32_t o[32];
            tmem_ld32(t_o + (uint32_t)(cc * 32), o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * corr);
            tmem_st32(t_o + (uint32_t)(cc * 32), o);
          }
        }
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[t]);
      }
      if (!ok) break;
      // epilogue: O / l -> bf16 and lse.  The next unit's first P.V, which overwrites O, waits for
      // the p_full arrival that follows these reads.
      if (!bounded_wait_warp(&pv_done[t], (c - 1) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* orow = out + (size_t)(b * S + q_pos) * E + h * DH;
#pragma unroll 1
      for (int cc = 0; cc < DH / 32; ++cc) {
        uint32_t o[32];
        tmem_ld32(t_o + (uint32_t)(cc * 32), o);
        tmem_ld_wait();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16(__uint_as_float(o[q * 8 + 0]) * inv, __uint_as_float(o[q * 8 + 1]) * inv);
          w.y = pack_bf16(__uint_as_float(o[q * 8 + 2]) * inv, __uint_as_float(o[q * 8 + 3]) * inv);
          w.z = pack_bf16(__uint_as_float(o[q * 8 + 4]) * inv, __uint_as_float(o[q * 8 + 5]) * inv);
          w.w = pack_bf16(__uint_as_float(o[q * 8 + 6]) * inv, __uint_as_float(o[q * 8 + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + cc * 32 + q * 8) = w;
        }
      }
      lse[(size_t)bh * S + q_pos] = (m + log2f(l)) * 0.6931471805599453f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}


// ============================================================== backward

// Persistent: one CTA per SM walks work units (batch, head, 128-key block), the units with the most
// query blocks first, in snake order over the CTAs.  A unit walks its query blocks from the diagonal
// to the end of the sequence, and the CTA's blocks form one pipeline across units: the next unit's
// K / V and first Q / dO stages load, and its first S^T / dP^T are computed, while the last block of
// the previous unit is still in flight.  The softmax warps write a finished unit's last dQ and its
// dK / dV right after the next unit's first block (releasing TMEM before storing), so they never
// wait for a unit's last products.  Per query block i:
//   MMA:     S^T = K Q_i^T, dP^T = V dO_i^T                                      (TMEM, fp32)
//   softmax: P^T = exp2(S^T * scale_log2 - lse2[q]) with the causal mask, dS^T = P^T (dP^T - D[q]);
//            P^T goes back to TMEM as bf16 (A operand of dV), dS^T to shared memory
//   MMA:     dV += P^T dO_i   (A from TMEM)
//            dK += dS^T Q_i   (A = dS^T in shared memory, K-major)
//            dQ_i = dS K      (A = the same dS^T read MN-major, B = K MN-major)
//   dQ_i:    TMEM -> one swizzled [32][32] shared box per softmax warp -> TMA reduce-add into the
//            fp32 accumulator ([B, H, S, Dh]), done by each softmax warp on its own one block later
// The tensor core and the softmax warps overlap across blocks: as soon as the softmax warps hold
// S^T / dP^T of block i in registers (sd_used), the MMA warp issues S^T / dP^T of block i+1; once
// P^T / dS^T of block i are written (ds_ready) it issues dV / dK / dQ of block i, while the softmax
// warps read out dQ of block i-1 and start on block i+1.  Only the writes of P^T (TMEM) and dS^T
// (shared memory) of block i+1 wait for block i's MMAs to finish reading them.  Q / dO run in three
// stages, so their loads are issued two blocks ahead.
// TMEM columns: S^T [0,128), dP^T [128,256), dV [256,320), dK [320,384), dQ [384,448), P^T [448,512).
// Eight softmax warps: warps w and w+4 share the TMEM lanes of quadrant w % 4 and split the 128
// query columns into halves.  The per-query rows nl = -lse*log2(e) and D = rowsum(dO*O) arrive by
// bulk copy with Q_i / dO_i.  A unit's dK (times the softmax scale, rotated back by RoPE when tables
// are given) and dV leave by TMA store to the packed gradient buffer; dQ's scale and inverse RoPE
// are applied by the caller's post pass.
namespace bwd {
constexpr int NSOFT = 8;
// Warpgroup 0: warp 0 TMA, warp 1 MMA, warps 2-3 idle; warps 4.. softmax.  (Registers are granted
// per warpgroup, so the two idle warps cost none; moving registers from warpgroup 0 to the softmax
// warps with setmaxnreg measured slower.)
constexpr int THREADS_B = 128 + 32 * NSOFT;
// With a dedicated readout warpgroup (the kernel's DQW form), warps 12-15 take every TMEM readout
// off the softmax warps: each block's dQ (staged and added into the fp32 accumulator) and a finished
// unit's dK / dV (stored as bf16), one TMEM lane quadrant per warp.  The softmax warps then only
// compute and write P^T / dS^T.  The 512 threads launch at 128 registers each (65,536 per block);
// warpgroup 0 and the readout warpgroup give registers up with setmaxnreg and the two softmax
// warpgroups take them, and the four shares add up to the launch total.
constexpr int THREADS_BQ = 512;
constexpr int REG_WG0 = 96, REG_SOFT = 160, REG_OUT = 96;
// (registers per warpgroup share x 128 threads) summed == 128 registers per thread x 512 threads
static_assert((REG_WG0 + 2 * REG_SOFT + REG_OUT) * 128 == 128 * THREADS_BQ, "register shares = launch total");
constexpr int WPQ = NSOFT / 4;              // softmax warps per TMEM lane quadrant
constexpr int QCOLS = BQ / WPQ;             // query columns (of S^T / dP^T) per softmax warp
constexpr int DCOLS = D / WPQ;              // head-dim columns (of dQ / dK / dV) per softmax warp
// The dQ / dK / dV staging area (SM_DQ, DQ_BYTES) holds one 4 KB box per softmax warp, and the boxes
// are 32 columns wide: both are laid out for exactly eight softmax warps (32 head-dim columns each).
static_assert(NSOFT == 8 && DCOLS == 32 && NSOFT * 4096 == BQ * D * 4, "staging laid out for 8 softmax warps");
constexpr int QST = 3;                               // Q / dO / row-vector stages (loads run two blocks ahead)
// K is double buffered (the next unit's key block loads while this one finishes); V has one buffer,
// which its last reader (the unit's last dP^T) releases early in the unit's last block.
constexpr int SM_K = 0, SM_V = 2 * TILE_BYTES, SM_Q = 3 * TILE_BYTES, SM_DO = SM_Q + QST * TILE_BYTES;
constexpr int SM_DS = SM_DO + QST * TILE_BYTES;
constexpr int DQ_BYTES = BQ * D * 4;                 // the fp32 dQ tile: two [128][32] boxes, 128-byte swizzle
constexpr int SM_DQ = SM_DS + 2 * TILE_BYTES;
constexpr int VEC_BYTES = 2 * BQ * 4;                // nl[128], D[128] of one query block
constexpr int SM_VEC = SM_DQ + DQ_BYTES;             // [QST] stages
constexpr int SM_BAR = SM_VEC + QST * VEC_BYTES;
constexpr int SMEM_TOTAL = SM_BAR + 256 + 1024;
static_assert(SMEM_TOTAL <= 227 * 1024, "shared memory");
constexpr uint32_t C_S = 0, C_DP = 128, C_DV = 256, C_DK = 320, C_DQ = 384, C_P = 448;
constexpr uint32_t IDESC_SD = make_idesc(1, 128, 128, 0, 0);  // K Q^T / V dO^T: both K-major
constexpr uint32_t IDESC_VK = make_idesc(1, 128, 64, 0, 1);   // dV / dK: A (TMEM or K-major), B MN-major
constexpr uint32_t IDESC_Q = make_idesc(1, 128, 64, 1, 1);    // dQ: A MN-major (dS^T), B MN-major (K)

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

template <int N> __device__ __forceinline__ void tmem_ld_n(uint32_t taddr, uint32_t (&r)[N]) {
  static_assert(N == 16 || N == 32, "columns");
  if constexpr (N == 32) tmem_ld32(taddr, r);
  else tmem_ld16(taddr, r);
}
template <int N> __device__ __forceinline__ void tmem_st_n(uint32_t taddr, const uint32_t (&r)[N]) {
  static_assert(N == 16 || N == 32, "columns");
  if constexpr (N == 32) tmem_st32(taddr, r);
  else tmem_st16(taddr, r);
}

template <bool DQW>
__global__ void __launch_bounds__(DQW ? THREADS_BQ : THREADS_B, 1)
    fa_bwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                     const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dk,
                     const __grid_constant__ CUtensorMap tm_dv,
                     const float* __restrict__ nl_g,
                     const float* __restrict__ Dsum,
                     const float* __restrict__ rope_cos,
                     const float* __restrict__ rope_sin, int* __restrict__ unit_ctr, int S, int H, int nunits,
                     int hgroup, float scale, float scale_log2) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SM_BAR);
  uint64_t* k_full = bar + 0;          // [2] K buffers (alternate work units)
  uint64_t* k_empty = bar + 2;         // [2] the unit's last dQ product has retired
  uint64_t* v_full = bar + 4;
  uint64_t* v_empty = bar + 5;         // the unit's last dP^T product has retired
  uint64_t* q_full = bar + 6;          // [QST]
  uint64_t* q_empty = bar + 6 + QST;   // [QST]
  uint64_t* sd_full = bar + 6 + 2 * QST;
  uint64_t* ds_ready = sd_full + 1;
  uint64_t* mm_done = sd_full + 2;
  uint64_t* dq_free = sd_full + 3;
  uint64_t* drain = sd_full + 4;       // final commit: every MMA of this CTA has retired
  uint64_t* sd_used = sd_full + 5;     // the softmax warps have loaded S^T / dP^T into registers
  uint64_t* dkv_free = sd_full + 6;    // the softmax warps have read dK / dV of the unit out of TMEM
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sd_full + 7);
  const UnitFeed feed{sd_full + 8, sd_full + 8 + UNIT_RING, reinterpret_cast<volatile int*>(sd_full + 8 + 2 * UNIT_RING)};
  static_assert((6 + 2 * QST + 8 + 2 * UNIT_RING) * 8 + UNIT_RING * 4 <= 256, "barrier area");

  const int E = H * D;
  const int nk = S / BKV;
  const int nbh = nunits / nk;
  const int G = (int)gridDim.x, cta = (int)blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // Work unit u = (key block kb, batch-head bh), key-block-major so the units with the most query
  // blocks come first; the CTA's units come from the unit feed.  The CTA's blocks form one flat
  // sequence: unit k of this CTA contributes query blocks kb .. nk-1.
  struct Unit {
    int kb, bh, niter;
  };
  auto decode = [&](int u) -> Unit {
    if (u < 0 || u >= nunits) return Unit{0, 0, 0};
    int kb, bh;
    bwd_unit_coords(u, nk, nbh, hgroup, &kb, &bh);
    return Unit{kb, bh, nk - kb};
  };
  // every reader warp calls this once for k = 0, 1, ... up to the first unit with niter == 0
  auto unit_of = [&](int k) -> Unit { return decode(feed.get(k)); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int i = 0; i < QST; ++i) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], 1); }
    mbar_init(sd_full, 1);
    mbar_init(ds_ready, 32 * NSOFT);
    mbar_init(mm_done, 1);
    mbar_init(dq_free, DQW ? 128 : 32 * NSOFT);
    mbar_init(drain, 1);
    mbar_init(sd_used, 32 * NSOFT);
    mbar_init(dkv_free, DQW ? 128 : 32 * NSOFT);
    for (int i = 0; i < UNIT_RING; ++i) {
      mbar_init(&feed.full[i], 1);
      mbar_init(&feed.empty[i], 1 + NSOFT + (DQW ? 4 : 0));  // MMA warp, softmax warps, readout warps
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
    tma_prefetch_desc(&tm_dk);
    tma_prefetch_desc(&tm_dv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  // Roles by warpgroup; in the DQW form each warpgroup first takes its register share (one
  // setmaxnreg per warpgroup, inside its own branch, so no other role's values are live across it).
  if (warp < 4) {
    if constexpr (DQW) setmaxnreg_dec<REG_WG0>();
    if (warp == 0) {
      // ------------------------------------------------------------ TMA producer
      // Per unit: K into buffer k & 1 (once the unit two back has finished with it), then the unit's
      // first Q / dO / row-vector stage, then V (once the previous unit's last dP^T has read the single
      // V buffer), then the remaining stages.  This is the order in which the slots drain.
      if (lane == 0) {
        uint32_t n = 0, nkl = 0, nvl = 0;  // Q stages, K and V tiles issued
        bool ok = true;
        int u = cta;
        for (int k = 0; ok; ++k) {
          if (!feed.put(k, u)) break;
          const Unit un = decode(u);
          if (un.niter == 0) break;
          const int u_next = min(feed.draw(G, unit_ctr), nunits);
          const int b = un.bh / H, h = un.bh % H;
          const int krow = b * S + un.kb * BKV;
          const size_t row_base = (size_t)un.bh * S;
          const int kbuf = k & 1;
          if (!bounded_wait(&k_empty[kbuf], ((k >> 1) & 1) ^ 1u, DEV_TIMEOUT_ATTN)) break;
          mbar_arrive_expect_tx(&k_full[kbuf], TILE_BYTES);
          tma_load_2d(smem + SM_K + kbuf * TILE_BYTES, &tm_k, &k_full[kbuf], h * D, krow);
          ++nkl;
          for (int i = 0; i < un.niter; ++i, ++n) {
            const uint32_t st = n % QST;
            if (!bounded_wait(&q_empty[st], ((n / QST) & 1) ^ 1u, DEV_TIMEOUT_ATTN)) { ok = false; break; }
            mbar_arrive_expect_tx(&q_full[st], 2 * TILE_BYTES + VEC_BYTES);
            const int qb = un.kb + i;
            const int qrow = b * S + qb * BQ;
            tma_load_2d(smem + SM_Q + st * TILE_BYTES, &tm_q, &q_full[st], h * D, qrow);
            tma_load_2d(smem + SM_DO + st * TILE_BYTES, &tm_do, &q_full[st], h * D, qrow);
            float* vec = reinterpret_cast<float*>(smem + SM_VEC + st * VEC_BYTES);
            bulk_load(vec, nl_g + row_base + (size_t)qb * BQ, BQ * 4, &q_full[st]);
            bulk_load(vec + BQ, Dsum + row_base + (size_t)qb * BQ, BQ * 4, &q_full[st]);
            if (i == 0) {
              if (!bounded_wait(v_empty, (k & 1) ^ 1u, DEV_TIMEOUT_ATTN)) { ok = false; ++n; break; }
              mbar_arrive_expect_tx(v_full, TILE_BYTES);
              tma_load_2d(smem + SM_V, &tm_v, v_full, h * D, krow);
              ++nvl;
            }
          }
          u = u_next;
        }
        // no copy may still be landing in shared memory when the CTA exits: the last load of every
        // slot has completed (the consumers waited for all of them on the normal path)
        for (uint32_t k = nkl > 2u ? nkl - 2 : 0; k < nkl; ++k)
          bounded_wait(&k_full[k & 1], (k >> 1) & 1, DEV_TIMEOUT_ATTN);
        if (nvl > 0) bounded_wait(v_full, (nvl - 1) & 1, DEV_TIMEOUT_ATTN);
        for (uint32_t j = n > (uint32_t)QST ? n - QST : 0; j < n; ++j)
          bounded_wait(&q_full[j % QST], (j / QST) & 1, DEV_TIMEOUT_ATTN);
      }
    } else if (warp == 1) {
      // ------------------------------------------------------------ MMA issuer
      const uint32_t sv = smem_u32(smem + SM_V), sds = smem_u32(smem + SM_DS);
      struct Cur {
        int k;      // unit of this CTA
        Unit un;
        int i;      // query block inside the unit (query block kb + i)
        uint32_t n; // block of the CTA's flat sequence
      };
      auto advance = [&](Cur c) -> Cur {
        if (++c.i == c.un.niter) {
          ++c.k;
          c.un = unit_of(c.k);
          c.i = 0;
        }
        ++c.n;
        return c;
      };
      // S^T / dP^T of block c -> sd_full; the unit's last one also releases V
      auto issue_sd = [&](const Cur& c) -> bool {
        const uint32_t st = c.n % QST;
        if (!bounded_wait_warp(&q_full[st], (c.n / QST) & 1, DEV_TIMEOUT_ATTN)) return false;
        if (c.i == 0) {
          if (!bounded_wait_warp(&k_full[c.k & 1], (c.k >> 1) & 1, DEV_TIMEOUT_ATTN)) return false;
          if (!bounded_wait_warp(v_full, c.k & 1, DEV_TIMEOUT_ATTN)) return false;
        }
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + SM_K + (c.k & 1) * TILE_BYTES);
        const uint32_t sq = smem_u32(smem + SM_Q + st * TILE_BYTES);
        const uint32_t sdo = smem_u32(smem + SM_DO + st * TILE_BYTES);
  #pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          umma_f16_w(tmem + C_S, smem_desc_sw128(sk + k * 32, 16, 1024), smem_desc_sw128(sq + k * 32, 16, 1024),
                     IDESC_SD, k > 0 ? 1u : 0u);
          umma_f16_w(tmem + C_DP, smem_desc_sw128(sv + k * 32, 16, 1024), smem_desc_sw128(sdo + k * 32, 16, 1024),
                     IDESC_SD, k > 0 ? 1u : 0u);
        }
        umma_commit_w(sd_full);
        if (c.i == c.un.niter - 1) umma_commit_w(v_empty);
        return true;
      };
      Cur cur{0, unit_of(0), 0, 0};
      bool ok = cur.un.niter > 0 && issue_sd(cur);
      while (ok && cur.un.niter > 0) {
        const Cur nxt = advance(cur);
        if (nxt.un.niter > 0) {
          // the softmax warps hold S^T / dP^T of this block in registers: the next block (of this
          // unit or the next) can overwrite them
          if (!bounded_wait_warp(sd_used, cur.n & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
          if (!issue_sd(nxt)) { ok = false; break; }
        }
        // softmax of this block is done: P^T (TMEM) and dS^T (smem) are ready
        if (!bounded_wait_warp(ds_ready, cur.n & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        // a unit's first dV / dK products overwrite the accumulators: the previous unit's must be read
        if (cur.i == 0 && cur.k > 0 && !bounded_wait_warp(dkv_free, (cur.k - 1) & 1, DEV_TIMEOUT_ATTN)) {
          ok = false;
          break;
        }
        // dQ of the previous block has been read out of TMEM
        if (cur.n > 0 && !bounded_wait_warp(dq_free, (cur.n - 1) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        tc_fence_after();
        const uint32_t st = cur.n % QST;
        const uint32_t sq = smem_u32(smem + SM_Q + st * TILE_BYTES), sdo = smem_u32(smem + SM_DO + st * TILE_BYTES);
        const uint32_t sk = smem_u32(smem + SM_K + (cur.k & 1) * TILE_BYTES);
        // dV, dK and dQ are three independent accumulation chains, issued interleaved
  #pragma unroll
        for (int k = 0; k < BQ / 16; ++k) {  // 16 queries (dV, dK) / 16 keys (dQ) per MMA
          const uint32_t acc = (cur.i > 0 || k > 0) ? 1u : 0u;
          umma_f16_ts_w(tmem + C_DV, tmem + C_P + (uint32_t)(k * 8), smem_desc_sw128(sdo + k * 2048, TILE_BYTES, 1024),
                        IDESC_VK, acc);
          umma_f16_w(tmem + C_DK, smem_desc_sw128(sds + (k >> 2) * TILE_BYTES + (k & 3) * 32, 16, 1024),
                     smem_desc_sw128(sq + k * 2048, TILE_BYTES, 1024), IDESC_VK, acc);
          umma_f16_w(tmem + C_DQ, smem_desc_sw128(sds + k * 2048, TILE_BYTES, 1024),
                     smem_desc_sw128(sk + k * 2048, TILE_BYTES, 1024), IDESC_Q, k > 0 ? 1u : 0u);
        }
        umma_commit_w(mm_done);
        umma_commit_w(&q_empty[st]);
        if (cur.i == cur.un.niter - 1) umma_commit_w(&k_empty[cur.k & 1]);
        cur = nxt;
      }
      // TMEM is freed below only after every MMA issued here has retired
      umma_commit_w(drain);
      bounded_wait_warp(drain, 0, DEV_TIMEOUT_ATTN);
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------ softmax (P^T, dS^T)
    if constexpr (DQW) setmaxnreg_inc<REG_SOFT>();
    const int quarter = warp & 3;
    const int cs = (warp - 4) >> 2;               // column slice: queries [QCOLS*cs, +QCOLS), head dims [DCOLS*cs, +DCOLS)
    const int r_local = quarter * 32 + lane;      // key row (S^T / dP^T / dV / dK) and query row (dQ)
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    uint8_t* sds = smem + SM_DS;
    // This warp's 4 KB staging area: one [32][32] fp32 dQ box (128-byte swizzle), or the [32][32] bf16
    // dK and dV boxes (64-byte swizzle) of a finished unit.  The warps stage and store independently.
    const uint32_t stg = smem_u32(smem + SM_DQ) + (uint32_t)((cs * 4 + quarter) * 4096);
    bool ok = true;
    auto stage_free = [&]() {  // the warp's last bulk copy has read the staging area
      if (lane == 0) bulk_wait_read0();
      __syncwarp();
    };
    // dQ rows [quarter*32, +32), columns [cs*DCOLS, +DCOLS) of a block, out of TMEM (dq_free)
    auto dq_load = [&](uint32_t (&dq)[DCOLS]) {
      tc_fence_after();
      tmem_ld_n<DCOLS>(t_lane + C_DQ + (uint32_t)(cs * DCOLS), dq);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(dq_free);
    };
    // ... then staged and added into the fp32 accumulator; y = the block's first accumulator row
    auto dq_store = [&](const uint32_t (&dq)[DCOLS], int y) {
      stage_free();
#pragma unroll
      for (int k = 0; k < DCOLS / 4; ++k)
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(stg + lane * 128 + ((k ^ (lane & 7)) << 4)),
                     "r"(dq[k * 4]), "r"(dq[k * 4 + 1]), "r"(dq[k * 4 + 2]), "r"(dq[k * 4 + 3]));
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d_bulk(&tm_dq, stg, cs * DCOLS, y + quarter * 32);
        bulk_commit();
      }
    };
    // A finished unit: dQ of its last block, then dK (times the softmax scale, rotated back by RoPE
    // when tables are given) and dV.  Both TMEM regions are released before anything is stored.
    auto unit_out = [&](const Unit& pu, int y) {
      uint32_t dq[DCOLS], dk[DCOLS], dv[DCOLS];
      dq_load(dq);
      tmem_ld_n<DCOLS>(t_lane + C_DK + (uint32_t)(cs * DCOLS), dk);
      tmem_ld_n<DCOLS>(t_lane + C_DV + (uint32_t)(cs * DCOLS), dv);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(dkv_free);
      dq_store(dq, y);
      const int b = pu.bh / H, h = pu.bh % H;
      const int key = pu.kb * BKV + r_local;  // position of this thread's key
      stage_free();
#pragma unroll
      for (int q = 0; q < DCOLS / 8; ++q) {
        float x[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) x[t] = __uint_as_float(dk[q * 8 + t]) * scale;
        if (rope_cos) {  // the 4 rotation pairs of these 8 columns: one 16-byte load each
          const size_t pr = (size_t)key * (D / 2) + ((cs * DCOLS + q * 8) >> 1);
          const float4 c4 = __ldg(reinterpret_cast<const float4*>(rope_cos + pr));
          const float4 s4 = __ldg(reinterpret_cast<const float4*>(rope_sin + pr));
          const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float a0 = x[2 * t], a1 = x[2 * t + 1];
            x[2 * t] = a0 * cc[t] + a1 * ss[t];
            x[2 * t + 1] = -a0 * ss[t] + a1 * cc[t];
          }
        }
        const uint32_t off = (uint32_t)(lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4));
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(stg + off), "r"(pack_bf16(x[0], x[1])),
                     "r"(pack_bf16(x[2], x[3])), "r"(pack_bf16(x[4], x[5])), "r"(pack_bf16(x[6], x[7])));
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(stg + 2048 + off),
                     "r"(pack_bf16(__uint_as_float(dv[q * 8 + 0]), __uint_as_float(dv[q * 8 + 1]))),
                     "r"(pack_bf16(__uint_as_float(dv[q * 8 + 2]), __uint_as_float(dv[q * 8 + 3]))),
                     "r"(pack_bf16(__uint_as_float(dv[q * 8 + 4]), __uint_as_float(dv[q * 8 + 5]))),
                     "r"(pack_bf16(__uint_as_float(dv[q * 8 + 6]), __uint_as_float(dv[q * 8 + 7]))));
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const int y0 = b * S + pu.kb * BKV + quarter * 32;
        tma_store_2d_bulk(&tm_dk, stg, h * D + cs * DCOLS, y0);
        tma_store_2d_bulk(&tm_dv, stg + 2048, h * D + cs * DCOLS, y0);
        bulk_commit();
      }
    };
    uint32_t n = 0;        // block of the CTA's flat sequence
    int prev_y = 0;        // dQ accumulator row of block n-1
    Unit pu{0, 0, 0};      // the previous unit (its dK / dV stay in TMEM until its first successor block)
    for (int ku = 0;; ++ku) {
      const Unit un = unit_of(ku);
      if (un.niter == 0) break;
      for (int i = 0; i < un.niter; ++i, ++n) {
        const float* vec = reinterpret_cast<const float*>(smem + SM_VEC + (n % QST) * VEC_BYTES);
        const bool diag = (i == 0);
        ok = ok && bounded_wait_warp(sd_full, n & 1, DEV_TIMEOUT_ATTN);
        if (ok) {
          tc_fence_after();
          // P^T / dS^T of this thread's queries are computed into registers first (sub-chunks of 16;
          // the TMEM loads of sub-chunk g+1 are in flight while g is computed), and only then does
          // the thread wait for the previous block's MMAs to release the P^T columns and dS^T buffer.
          auto chunks = [&](auto diag_tag) {
            constexpr bool DIAG = decltype(diag_tag)::value;
            constexpr int NG = QCOLS / 16;          // sub-chunks of 16 queries
            // with two softmax warps per sub-partition the TMEM loads of sub-chunk g+1 are issued
            // before g is computed; with four, the other warps hide the load latency instead
            constexpr bool PREFETCH = (WPQ == 2);
            constexpr int NB = PREFETCH ? 2 : 1;
            uint32_t rs[NB][16], rd[NB][16];
            uint32_t pp[QCOLS / 2], dd[QCOLS / 2];
            const uint32_t c0 = (uint32_t)(cs * QCOLS);
            const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
            if constexpr (PREFETCH) {
              tmem_ld16(t_lane + C_S + c0, rs[0]);
              tmem_ld16(t_lane + C_DP + c0, rd[0]);
              tmem_ld_wait();
            }
#pragma unroll
            for (int g = 0; g < NG; ++g) {
              const int bb = PREFETCH ? (g & 1) : 0;
              if constexpr (PREFETCH) {
                if (g + 1 < NG) {
                  tmem_ld16(t_lane + C_S + c0 + (uint32_t)((g + 1) * 16), rs[(g + 1) & 1]);
                  tmem_ld16(t_lane + C_DP + c0 + (uint32_t)((g + 1) * 16), rd[(g + 1) & 1]);
                }
              } else {
                tmem_ld16(t_lane + C_S + c0 + (uint32_t)(g * 16), rs[0]);
                tmem_ld16(t_lane + C_DP + c0 + (uint32_t)(g * 16), rd[0]);
                tmem_ld_wait();
              }
              const int q0 = cs * QCOLS + g * 16;  // first query of the sub-chunk
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                const float4 nl4 = *reinterpret_cast<const float4*>(vec + q0 + j);
                const float4 d4 = *reinterpret_cast<const float4*>(vec + BQ + q0 + j);
                const float nlv[4] = {nl4.x, nl4.y, nl4.z, nl4.w};
                const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
                float p[4], d[4];
#pragma unroll
                for (int t = 0; t < 4; t += 2) {  // two queries per paired fp32 instruction
                  float x0, x1;
                  f2_unpack(fma2(f2_pack(__uint_as_float(rs[bb][j + t]), __uint_as_float(rs[bb][j + t + 1])), sc2,
                                 f2_pack(nlv[t], nlv[t + 1])), x0, x1);
                  p[t] = fast_exp2(x0);
                  p[t + 1] = fast_exp2(x1);
                  if (DIAG && r_local > q0 + j + t) p[t] = 0.f;
                  if (DIAG && r_local > q0 + j + t + 1) p[t + 1] = 0.f;
                  f2_unpack(mul2(f2_pack(p[t], p[t + 1]),
                                 sub2(f2_pack(__uint_as_float(rd[bb][j + t]), __uint_as_float(rd[bb][j + t + 1])),
                                      f2_pack(dv[t], dv[t + 1]))),
                            d[t], d[t + 1]);
                }
                pp[g * 8 + (j >> 1)] = pack_bf16(p[0], p[1]);
                pp[g * 8 + (j >> 1) + 1] = pack_bf16(p[2], p[3]);
                dd[g * 8 + (j >> 1)] = pack_bf16(d[0], d[1]);
                dd[g * 8 + (j >> 1) + 1] = pack_bf16(d[2], d[3]);
              }
              if constexpr (PREFETCH) {
                if (g + 1 < NG) tmem_ld_wait();
                if (g == NG - 2) {  // the last sub-chunk has landed: S^T / dP^T may be overwritten
                  tc_fence_before();
                  mbar_arrive(sd_used);
                }
              }
            }
            if constexpr (!PREFETCH) {
              tc_fence_before();
              mbar_arrive(sd_used);
            }
            if (n > 0) {
              // the previous block's dV / dK / dQ MMAs have finished reading P^T and dS^T
              ok = bounded_wait_warp(mm_done, (n - 1) & 1, DEV_TIMEOUT_ATTN);
              if (!ok) return;
              tc_fence_after();
            }
            tmem_st_n<QCOLS / 2>(t_lane + C_P + (uint32_t)(cs * (QCOLS / 2)), pp);
            // dS^T row segment -> shared memory in the swizzled [q-half][key][64] layout
            uint8_t* rowp = sds + ((cs * QCOLS) >> 6) * TILE_BYTES + r_local * 128;
            const int t0 = ((cs * QCOLS) & 63) >> 3;
#pragma unroll
            for (int t = 0; t < QCOLS / 8; ++t)
              *reinterpret_cast<uint4*>(rowp + (((t0 + t) ^ (r_local & 7)) * 16)) =
                  make_uint4(dd[t * 4], dd[t * 4 + 1], dd[t * 4 + 2], dd[t * 4 + 3]);
          };
          if (diag) chunks(std::integral_constant<bool, true>{});
          else chunks(std::integral_constant<bool, false>{});
          if (ok) {
            tmem_st_wait();
            tc_fence_before();
            fence_async_smem();
            mbar_arrive(ds_ready);
          }
        }
        if (!DQW && ok && n > 0) {
          // the previous block's dQ; at a unit's first block, also the previous unit's dK / dV (the
          // MMA warp waits for both before this block's products)
          if (i > 0) {
            uint32_t dq[DCOLS];
            dq_load(dq);
            dq_store(dq, prev_y);
          } else {
            unit_out(pu, prev_y);
          }
        }
        prev_y = (int)((size_t)un.bh * S + (size_t)(un.kb + i) * BQ);
      }
      pu = un;
      if (!ok) break;
    }
    if constexpr (!DQW) {
      if (n > 0 && ok && bounded_wait_warp(mm_done, (n - 1) & 1, DEV_TIMEOUT_ATTN)) unit_out(pu, prev_y);
      if (lane == 0) bulk_wait0();  // every dQ reduction and dK / dV store of this warp has landed
    }
  } else if constexpr (DQW) {
    // ------------------------------------------------------------ TMEM readout (DQW form)
    setmaxnreg_dec<REG_OUT>();
    // Warp 12 + q reads TMEM lanes [32 q, 32 q + 32): after each block's products, the block's dQ rows
    // (all 64 head dims) go through two [32][32] fp32 boxes (128-byte swizzle) into the accumulator by
    // TMA reduce-add; after a unit's last block, its dK (times the softmax scale, rotated back by RoPE
    // when tables are given) and dV rows leave as four [32][32] bf16 boxes (64-byte swizzle) by TMA
    // store.  dq_free / dkv_free are arrived as soon as the TMEM columns have been read.
    const int quarter = warp & 3;
    const int r_local = quarter * 32 + lane;  // query row of dQ, key row of dK / dV
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    const uint32_t stg = smem_u32(smem + SM_DQ) + (uint32_t)(quarter * 8192);  // this warp's 8 KB
    auto stage_free = [&]() {  // the warp's last bulk copy has read the staging area
      if (lane == 0) bulk_wait_read0();
      __syncwarp();
    };
    bool ok = true;
    uint32_t n = 0;
    for (int ku = 0; ok; ++ku) {
      const Unit un = unit_of(ku);
      if (un.niter == 0) break;
      const int b = un.bh / H, hd = un.bh % H;
      for (int i = 0; i < un.niter; ++i, ++n) {
        // off the critical path: the MMA warp needs this block's dq_free only after the next
        // block's softmax, so the wait sleeps between polls
        if (!bounded_wait_warp_sleep(mm_done, n & 1, DEV_TIMEOUT_ATTN, 100)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int part = 0; part < 4; ++part) {  // head dims [16 part, 16 part + 16)
          uint32_t dq[16];
          tmem_ld16(t_lane + C_DQ + (uint32_t)(part * 16), dq);
          tmem_ld_wait();
          if (part == 3) {
            tc_fence_before();
            mbar_arrive(dq_free);
          }
          if (part == 0) stage_free();
          // box part / 2 ([32 rows][32 dims] fp32, 128-byte swizzle), 16-byte chunks 4 (part & 1) ..
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const int k = (part & 1) * 4 + j;
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};"
                         ::"r"(stg + (uint32_t)((part >> 1) * 4096 + lane * 128 + ((k ^ (lane & 7)) << 4))),
                         "r"(dq[j * 4]), "r"(dq[j * 4 + 1]), "r"(dq[j * 4 + 2]), "r"(dq[j * 4 + 3]));
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          const int y = (int)((size_t)un.bh * S + (size_t)(un.kb + i) * BQ) + quarter * 32;
          tma_reduce_add_2d_bulk(&tm_dq, stg, 0, y);
          tma_reduce_add_2d_bulk(&tm_dq, stg + 4096, 32, y);
          bulk_commit();
        }
        if (i == un.niter - 1) {
          const int key = un.kb * BKV + r_local;  // position of this thread's key
#pragma unroll
          for (int part = 0; part < 8; ++part) {  // 16 dims at a time: dK dims [0,64), then dV
            const bool is_k = part < 4;
            const int c0 = (part & 3) * 16;
            uint32_t x[16];
            tmem_ld16(t_lane + (is_k ? C_DK : C_DV) + (uint32_t)c0, x);
            tmem_ld_wait();
            if (part == 7) {
              tc_fence_before();
              mbar_arrive(dkv_free);
            }
            if (part == 0) stage_free();  // the dQ reduce-adds above have read the staging area
            // [32 rows][32 dims] boxes: dK [0,32) at +0, dK [32,64) at +2048, dV likewise at +4096
            const uint32_t box = stg + (uint32_t)((part >> 1) * 2048);
#pragma unroll
            for (int h2 = 0; h2 < 2; ++h2) {  // 8 dims per 16-byte chunk
              const int q = (part & 1) * 2 + h2;  // chunk inside the 32-dim box
              float v[8];
#pragma unroll
              for (int t = 0; t < 8; ++t) v[t] = __uint_as_float(x[h2 * 8 + t]);
              if (is_k) {
#pragma unroll
                for (int t = 0; t < 8; ++t) v[t] *= scale;
                if (rope_cos) {  // the 4 rotation pairs of these 8 dims: one 16-byte load each
                  const size_t pr = (size_t)key * (D / 2) + ((c0 + h2 * 8) >> 1);
                  const float4 c4 = __ldg(reinterpret_cast<const float4*>(rope_cos + pr));
                  const float4 s4 = __ldg(reinterpret_cast<const float4*>(rope_sin + pr));
                  const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                  for (int t = 0; t < 4; ++t) {
                    const float a0 = v[2 * t], a1 = v[2 * t + 1];
                    v[2 * t] = a0 * cc[t] + a1 * ss[t];
                    v[2 * t + 1] = -a0 * ss[t] + a1 * cc[t];
                  }
                }
              }
              const uint32_t off = (uint32_t)(lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4));
              asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(box + off), "r"(pack_bf16(v[0], v[1])),
                           "r"(pack_bf16(v[2], v[3])), "r"(pack_bf16(v[4], v[5])), "r"(pack_bf16(v[6], v[7])));
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            const int y0 = b * S + un.kb * BKV + quarter * 32;
            tma_store_2d_bulk(&tm_dk, stg, hd * D, y0);
            tma_store_2d_bulk(&tm_dk, stg + 2048, hd * D + 32, y0);
            tma_store_2d_bulk(&tm_dv, stg + 4096, hd * D, y0);
            tma_store_2d_bulk(&tm_dv, stg + 6144, hd * D + 32, y0);
            bulk_commit();
          }
        }
      }
    }
    if (lane == 0) bulk_wait0();  // every dQ reduction and dK / dV store of this warp has landed
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
}  // namespace bwd

// ============================================================== backward, head dim 128
// The same pipeline as the head-dim-64 backward (work units, barriers, warp roles), with the products
// shaped for 128 head dims.  TMEM cannot hold 128-column S^T / dP^T next to 128-column dV / dK
// accumulators, so a block is 128 keys x 64 queries and dQ is computed transposed:
//   S^T = K Q_i^T, dP^T = V dO_i^T      M = 128 keys,      N = 64 queries, K = 128 head dims
//   dV += P^T dO_i (A from TMEM)        M = 128 keys,      N = 128 dims,   K = 64 queries
//   dK += dS^T Q_i (A = dS^T K-major)   M = 128 keys,      N = 128 dims,   K = 64 queries
//   dQ_i^T = K^T dS^T                   M = 128 head dims, N = 64 queries, K = 128 keys
//                                       (A = the K tile read MN-major, B = dS^T read MN-major)
// TMEM columns: S^T [0,64), dP^T [64,128), P^T [128,160), dQ^T [192,256), dV [256,384), dK [384,512).
// dQ^T comes out of TMEM with the head dims on the lanes; each softmax warp writes its [32 queries]
// [32 dims] piece transposed into its swizzled staging box (one conflict-free 4-byte store per query),
// so the fp32 accumulator keeps the [B, H, S, Dh] layout of the head-dim-64 kernel and the same post
// pass finishes dQ.  A key block meets the diagonal in query blocks 2 kb and 2 kb + 1, so the first
// two blocks of every unit are masked.  dK / dV of a finished unit leave as [32 keys][64 dims] bf16
// boxes by TMA store, dK first, through the warp's staging box.
namespace bwd128 {
using bwd::bulk_load;
using bwd::fence_async_smem;
constexpr int D = 128, BQ = 64, BKV = 128, NSOFT = 8;
constexpr int THREADS = 128 + 32 * NSOFT;  // warp 0 TMA, warp 1 MMA, warps 2-3 idle, warps 4-11 softmax
constexpr int QCOLS = 32;                  // queries per softmax warp (two warps per TMEM lane quadrant)
constexpr int DCOLS = 64;                  // head dims of dK / dV per softmax warp
constexpr int QST = 2;                     // Q / dO / row-vector stages
constexpr int KATOM = BKV * 128, QATOM = BQ * 128;  // one [rows][64] bf16 swizzle atom: 16 KB / 8 KB
constexpr int K_BYTES = 2 * KATOM, Q_BYTES = 2 * QATOM;
constexpr int SM_K = 0, SM_V = 2 * K_BYTES, SM_Q = SM_V + K_BYTES, SM_DO = SM_Q + QST * Q_BYTES;
constexpr int SM_DS = SM_DO + QST * Q_BYTES;  // dS^T [128 keys][64 queries] bf16: one atom
constexpr int SM_STG = SM_DS + KATOM;         // one 4 KB staging box per softmax warp
constexpr int VEC_BYTES = 2 * BQ * 4;         // nl[64], D[64] of one query block
constexpr int SM_VEC = SM_STG + NSOFT * 4096;
constexpr int SM_BAR = SM_VEC + QST * VEC_BYTES;
constexpr int SMEM_TOTAL = SM_BAR + 256 + 1024;
static_assert(SMEM_TOTAL <= 227 * 1024, "shared memory");
static_assert(NSOFT * QCOLS == 4 * BQ && NSOFT * DCOLS == 4 * D, "softmax warps cover a block");
constexpr uint32_t C_S = 0, C_DP = 64, C_P = 128, C_DQ = 192, C_DV = 256, C_DK = 384;
constexpr uint32_t IDESC_SD = make_idesc(1, 128, 64, 0, 0);   // S^T / dP^T: A, B K-major
constexpr uint32_t IDESC_VK = make_idesc(1, 128, 128, 0, 1);  // dV / dK: A TMEM or K-major, B MN-major
constexpr uint32_t IDESC_Q = make_idesc(1, 128, 64, 1, 1);    // dQ^T: A, B MN-major

__global__ void __launch_bounds__(THREADS, 1)
    fa_bwd_tc128_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                        const __grid_constant__ CUtensorMap tm_dq, const __grid_constant__ CUtensorMap tm_dk,
                        const __grid_constant__ CUtensorMap tm_dv, const float* __restrict__ nl_g,
                        const float* __restrict__ Dsum, const float* __restrict__ rope_cos,
                        const float* __restrict__ rope_sin, int* __restrict__ unit_ctr, int S, int H, int nunits,
                        int hgroup, float scale, float scale_log2) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw + 1023u) & ~1023u) - raw);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + SM_BAR);
  uint64_t* k_full = bar + 0;          // [2] K buffers (alternate work units)
  uint64_t* k_empty = bar + 2;         // [2] the unit's last dQ^T product has retired
  uint64_t* v_full = bar + 4;
  uint64_t* v_empty = bar + 5;         // the unit's last dP^T product has retired
  uint64_t* q_full = bar + 6;          // [QST]
  uint64_t* q_empty = bar + 6 + QST;   // [QST]
  uint64_t* sd_full = bar + 6 + 2 * QST;
  uint64_t* ds_ready = sd_full + 1;
  uint64_t* mm_done = sd_full + 2;
  uint64_t* dq_free = sd_full + 3;
  uint64_t* drain = sd_full + 4;       // final commit: every MMA of this CTA has retired
  uint64_t* sd_used = sd_full + 5;     // the softmax warps hold S^T / dP^T of the block in registers
  uint64_t* dkv_free = sd_full + 6;    // the softmax warps have read dK / dV of the unit out of TMEM
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(sd_full + 7);
  const UnitFeed feed{sd_full + 8, sd_full + 8 + UNIT_RING, reinterpret_cast<volatile int*>(sd_full + 8 + 2 * UNIT_RING)};
  static_assert((6 + 2 * QST + 8 + 2 * UNIT_RING) * 8 + UNIT_RING * 4 <= 256, "barrier area");

  const int E = H * D;
  const int nk = S / BKV;
  const int nbh = nunits / nk;
  const int G = (int)gridDim.x, cta = (int)blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // unit u = (key block kb, batch-head bh), key-block-major (most query blocks first), from the
  // unit feed
  struct Unit {
    int kb, bh, niter;
  };
  auto decode = [&](int u) -> Unit {
    if (u < 0 || u >= nunits) return Unit{0, 0, 0};
    int kb, bh;
    bwd_unit_coords(u, nk, nbh, hgroup, &kb, &bh);
    return Unit{kb, bh, 2 * (nk - kb)};
  };
  // every reader warp calls this once for k = 0, 1, ... up to the first unit with niter == 0
  auto unit_of = [&](int k) -> Unit { return decode(feed.get(k)); };

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) { mbar_init(&k_full[i], 1); mbar_init(&k_empty[i], 1); }
    mbar_init(v_full, 1);
    mbar_init(v_empty, 1);
    for (int i = 0; i < QST; ++i) { mbar_init(&q_full[i], 1); mbar_init(&q_empty[i], 1); }
    mbar_init(sd_full, 1);
    mbar_init(ds_ready, 32 * NSOFT);
    mbar_init(mm_done, 1);
    mbar_init(dq_free, 32 * NSOFT);
    mbar_init(drain, 1);
    mbar_init(sd_used, 32 * NSOFT);
    mbar_init(dkv_free, 32 * NSOFT);
    for (int i = 0; i < UNIT_RING; ++i) {
      mbar_init(&feed.full[i], 1);
      mbar_init(&feed.empty[i], 1 + NSOFT);  // MMA warp, softmax warps
    }
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
    tma_prefetch_desc(&tm_do);
    tma_prefetch_desc(&tm_dq);
    tma_prefetch_desc(&tm_dk);
    tma_prefetch_desc(&tm_dv);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t n = 0, nkl = 0, nvl = 0;
      bool ok = true;
      int u = cta;
      for (int k = 0; ok; ++k) {
        if (!feed.put(k, u)) break;
        const Unit un = decode(u);
        if (un.niter == 0) break;
        const int u_next = min(feed.draw(G, unit_ctr), nunits);
        const int b = un.bh / H, h = un.bh % H;
        const int krow = b * S + un.kb * BKV;
        const size_t row_base = (size_t)un.bh * S;
        const int kbuf = k & 1;
        if (!bounded_wait(&k_empty[kbuf], ((k >> 1) & 1) ^ 1u, DEV_TIMEOUT_ATTN)) break;
        mbar_arrive_expect_tx(&k_full[kbuf], K_BYTES);
        for (int a = 0; a < 2; ++a)
          tma_load_2d(smem + SM_K + kbuf * K_BYTES + a * KATOM, &tm_k, &k_full[kbuf], h * D + a * 64, krow);
        ++nkl;
        for (int i = 0; i < un.niter; ++i, ++n) {
          const uint32_t st = n % QST;
          if (!bounded_wait(&q_empty[st], ((n / QST) & 1) ^ 1u, DEV_TIMEOUT_ATTN)) { ok = false; break; }
          mbar_arrive_expect_tx(&q_full[st], 2 * Q_BYTES + VEC_BYTES);
          const int qb = 2 * un.kb + i;
          const int qrow = b * S + qb * BQ;
          for (int a = 0; a < 2; ++a) {
            tma_load_2d(smem + SM_Q + st * Q_BYTES + a * QATOM, &tm_q, &q_full[st], h * D + a * 64, qrow);
            tma_load_2d(smem + SM_DO + st * Q_BYTES + a * QATOM, &tm_do, &q_full[st], h * D + a * 64, qrow);
          }
          float* vec = reinterpret_cast<float*>(smem + SM_VEC + st * VEC_BYTES);
          bulk_load(vec, nl_g + row_base + (size_t)qb * BQ, BQ * 4, &q_full[st]);
          bulk_load(vec + BQ, Dsum + row_base + (size_t)qb * BQ, BQ * 4, &q_full[st]);
          if (i == 0) {
            if (!bounded_wait(v_empty, (k & 1) ^ 1u, DEV_TIMEOUT_ATTN)) { ok = false; ++n; break; }
            mbar_arrive_expect_tx(v_full, K_BYTES);
            for (int a = 0; a < 2; ++a)
              tma_load_2d(smem + SM_V + a * KATOM, &tm_v, v_full, h * D + a * 64, krow);
            ++nvl;
          }
        }
        u = u_next;
      }
      // no copy may still be landing in shared memory when the CTA exits
      for (uint32_t k = nkl > 2u ? nkl - 2 : 0; k < nkl; ++k)
        bounded_wait(&k_full[k & 1], (k >> 1) & 1, DEV_TIMEOUT_ATTN);
      if (nvl > 0) bounded_wait(v_full, (nvl - 1) & 1, DEV_TIMEOUT_ATTN);
      for (uint32_t j = n > (uint32_t)QST ? n - QST : 0; j < n; ++j)
        bounded_wait(&q_full[j % QST], (j / QST) & 1, DEV_TIMEOUT_ATTN);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t sv = smem_u32(smem + SM_V), sds = smem_u32(smem + SM_DS);
    struct Cur {
      int k;
      Unit un;
      int i;
      uint32_t n;
    };
    auto advance = [&](Cur c) -> Cur {
      if (++c.i == c.un.niter) {
        ++c.k;
        c.un = unit_of(c.k);
        c.i = 0;
      }
      ++c.n;
      return c;
    };
    auto issue_sd = [&](const Cur& c) -> bool {
      const uint32_t st = c.n % QST;
      if (!bounded_wait_warp(&q_full[st], (c.n / QST) & 1, DEV_TIMEOUT_ATTN)) return false;
      if (c.i == 0) {
        if (!bounded_wait_warp(&k_full[c.k & 1], (c.k >> 1) & 1, DEV_TIMEOUT_ATTN)) return false;
        if (!bounded_wait_warp(v_full, c.k & 1, DEV_TIMEOUT_ATTN)) return false;
      }
      tc_fence_after();
      const uint32_t sk = smem_u32(smem + SM_K + (c.k & 1) * K_BYTES);
      const uint32_t sq = smem_u32(smem + SM_Q + st * Q_BYTES);
      const uint32_t sdo = smem_u32(smem + SM_DO + st * Q_BYTES);
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {  // 16 head dims per MMA; atoms of 64 dims
        const uint32_t ka = (uint32_t)((k >> 2) * KATOM + (k & 3) * 32);
        const uint32_t qa = (uint32_t)((k >> 2) * QATOM + (k & 3) * 32);
        umma_f16_w(tmem + C_S, smem_desc_sw128(sk + ka, 16, 1024), smem_desc_sw128(sq + qa, 16, 1024), IDESC_SD,
                 k > 0 ? 1u : 0u);
        umma_f16_w(tmem + C_DP, smem_desc_sw128(sv + ka, 16, 1024), smem_desc_sw128(sdo + qa, 16, 1024), IDESC_SD,
                 k > 0 ? 1u : 0u);
      }
      umma_commit_w(sd_full);
      if (c.i == c.un.niter - 1) umma_commit_w(v_empty);
      return true;
    };
    Cur cur{0, unit_of(0), 0, 0};
    bool ok = cur.un.niter > 0 && issue_sd(cur);
    while (ok && cur.un.niter > 0) {
      const Cur nxt = advance(cur);
      if (nxt.un.niter > 0) {
        if (!bounded_wait_warp(sd_used, cur.n & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
        if (!issue_sd(nxt)) { ok = false; break; }
      }
      if (!bounded_wait_warp(ds_ready, cur.n & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
      if (cur.i == 0 && cur.k > 0 && !bounded_wait_warp(dkv_free, (cur.k - 1) & 1, DEV_TIMEOUT_ATTN)) {
        ok = false;
        break;
      }
      if (cur.n > 0 && !bounded_wait_warp(dq_free, (cur.n - 1) & 1, DEV_TIMEOUT_ATTN)) { ok = false; break; }
      tc_fence_after();
      const uint32_t st = cur.n % QST;
      const uint32_t sq = smem_u32(smem + SM_Q + st * Q_BYTES), sdo = smem_u32(smem + SM_DO + st * Q_BYTES);
      const uint32_t sk = smem_u32(smem + SM_K + (cur.k & 1) * K_BYTES);
      // dQ^T (16 keys per MMA) interleaved with dV and dK (16 queries per MMA)
#pragma unroll
      for (int j = 0; j < BKV / 16; ++j) {
        umma_f16_w(tmem + C_DQ, smem_desc_sw128(sk + j * 2048, KATOM, 1024), smem_desc_sw128(sds + j * 2048, KATOM, 1024),
                 IDESC_Q, j > 0 ? 1u : 0u);
        if (j < BQ / 16) {
          const uint32_t acc = (cur.i > 0 || j > 0) ? 1u : 0u;
          umma_f16_ts_w(tmem + C_DV, tmem + C_P + (uint32_t)(j * 8), smem_desc_sw128(sdo + j * 2048, QATOM, 1024),
                      IDESC_VK, acc);
          umma_f16_w(tmem + C_DK, smem_desc_sw128(sds + j * 32, 16, 1024), smem_desc_sw128(sq + j * 2048, QATOM, 1024),
                   IDESC_VK, acc);
        }
      }
      umma_commit_w(mm_done);
      umma_commit_w(&q_empty[st]);
      if (cur.i == cur.un.niter - 1) umma_commit_w(&k_empty[cur.k & 1]);
      cur = nxt;
    }
    umma_commit_w(drain);
    bounded_wait_warp(drain, 0, DEV_TIMEOUT_ATTN);
  } else if (warp >= 4) {
    const int quarter = warp & 3;
    const int cs = (warp - 4) >> 2;            // queries [32 cs, +32); head dims [64 cs, +64) of dK / dV
    const int r_local = quarter * 32 + lane;   // key row (S^T, dP^T, dV, dK); head dim row of dQ^T
    const uint32_t t_lane = tmem + ((uint32_t)(quarter * 32) << 16);
    uint8_t* sds = smem + SM_DS;
    const uint32_t stg = smem_u32(smem + SM_STG) + (uint32_t)((cs * 4 + quarter) * 4096);
    bool ok = true;
    auto stage_free = [&]() {
      if (lane == 0) bulk_wait_read0();
      __syncwarp();
    };
    // dQ^T rows (head dims) [32 quarter, +32), columns (queries) [32 cs, +32) of a block (dq_free)
    auto dq_load = [&](uint32_t (&dq)[32]) {
      tc_fence_after();
      tmem_ld32(t_lane + C_DQ + (uint32_t)(cs * 32), dq);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(dq_free);
    };
    // ... transposed into a [32 queries][32 dims] fp32 box (128-byte swizzle) and added into the
    // accumulator; y = the block's first accumulator row
    auto dq_store = [&](const uint32_t (&dq)[32], int y) {
      stage_free();
      const uint32_t col = (uint32_t)((lane & 3) * 4);
#pragma unroll
      for (int q = 0; q < 32; ++q)
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(stg + q * 128 + ((((uint32_t)lane >> 2) ^ (q & 7)) << 4) + col),
                     "r"(dq[q]));
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_reduce_add_2d_bulk(&tm_dq, stg, quarter * 32, y + cs * 32);
        bulk_commit();
      }
    };
    // 32 columns of dK (times the softmax scale, rotated back by RoPE when tables are given) or of dV,
    // packed to bf16 pairs
    auto pack_cols = [&](uint32_t col0, bool is_k, int key, uint32_t (&out)[16]) {
      uint32_t r[32];
      tmem_ld32(t_lane + (is_k ? C_DK : C_DV) + col0, r);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float x[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) x[t] = __uint_as_float(r[q * 8 + t]) * (is_k ? scale : 1.0f);
        if (is_k && rope_cos) {
          const size_t pr = (size_t)key * (D / 2) + ((col0 + q * 8) >> 1);
          const float4 c4 = __ldg(reinterpret_cast<const float4*>(rope_cos + pr));
          const float4 s4 = __ldg(reinterpret_cast<const float4*>(rope_sin + pr));
          const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const float a0 = x[2 * t], a1 = x[2 * t + 1];
            x[2 * t] = a0 * cc[t] + a1 * ss[t];
            x[2 * t + 1] = -a0 * ss[t] + a1 * cc[t];
          }
        }
#pragma unroll
        for (int t = 0; t < 4; ++t) out[q * 4 + t] = pack_bf16(x[2 * t], x[2 * t + 1]);
      }
    };
    // a [32 keys][64 dims] bf16 box (128-byte rows, swizzled) by TMA store
    auto store_box = [&](const CUtensorMap* map, const uint32_t (&p)[32], int x, int y) {
      stage_free();
#pragma unroll
      for (int c = 0; c < 8; ++c)
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(stg + lane * 128 + ((c ^ (lane & 7)) << 4)),
                     "r"(p[c * 4]), "r"(p[c * 4 + 1]), "r"(p[c * 4 + 2]), "r"(p[c * 4 + 3]));
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tma_store_2d_bulk(map, stg, x, y);
        bulk_commit();
      }
    };
    // A finished unit: dQ of its last block, then dK and dV; both TMEM regions are released before
    // anything is stored.
    auto unit_out = [&](const Unit& pu, int y) {
      uint32_t dq[32];
      dq_load(dq);
      const int key = pu.kb * BKV + r_local;
      uint32_t pk[32], pv[32];
      {
        uint32_t h0[16], h1[16];
        pack_cols((uint32_t)(cs * DCOLS), true, key, h0);
        pack_cols((uint32_t)(cs * DCOLS + 32), true, key, h1);
#pragma unroll
        for (int j = 0; j < 16; ++j) { pk[j] = h0[j]; pk[16 + j] = h1[j]; }
        pack_cols((uint32_t)(cs * DCOLS), false, key, h0);
        pack_cols((uint32_t)(cs * DCOLS + 32), false, key, h1);
#pragma unroll
        for (int j = 0; j < 16; ++j) { pv[j] = h0[j]; pv[16 + j] = h1[j]; }
      }
      tc_fence_before();
      mbar_arrive(dkv_free);
      dq_store(dq, y);
      const int b = pu.bh / H, h = pu.bh % H;
      const int y0 = b * S + pu.kb * BKV + quarter * 32;
      store_box(&tm_dk, pk, h * D + cs * DCOLS, y0);
      store_box(&tm_dv, pv, h * D + cs * DCOLS, y0);
    };
    uint32_t n = 0;
    int prev_y = 0;
    Unit pu{0, 0, 0};
    for (int ku = 0;; ++ku) {
      const Unit un = unit_of(ku);
      if (un.niter == 0) break;
      for (int i = 0; i < un.niter; ++i, ++n) {
        const float* vec = reinterpret_cast<const float*>(smem + SM_VEC + (n % QST) * VEC_BYTES);
        ok = ok && bounded_wait_warp(sd_full, n & 1, DEV_TIMEOUT_ATTN);
        if (ok) {
          tc_fence_after();
          // keys above the diagonal: key r_local against query moff + q of the block (blocks 0 and 1)
          const int moff = 64 * i;
          auto chunks = [&](auto diag_tag) {
            constexpr bool DIAG = decltype(diag_tag)::value;
            constexpr int NG = QCOLS / 16;
            uint32_t rs[2][16], rd[2][16];
            uint32_t pp[QCOLS / 2], dd[QCOLS / 2];
            const uint32_t c0 = (uint32_t)(cs * QCOLS);
            const uint64_t sc2 = f2_pack(scale_log2, scale_log2);
            tmem_ld16(t_lane + C_S + c0, rs[0]);
            tmem_ld16(t_lane + C_DP + c0, rd[0]);
            tmem_ld_wait();
#pragma unroll
            for (int g = 0; g < NG; ++g) {
              const int bb = g & 1;
              if (g + 1 < NG) {
                tmem_ld16(t_lane + C_S + c0 + (uint32_t)((g + 1) * 16), rs[(g + 1) & 1]);
                tmem_ld16(t_lane + C_DP + c0 + (uint32_t)((g + 1) * 16), rd[(g + 1) & 1]);
              }
              const int q0 = cs * QCOLS + g * 16;
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                const float4 nl4 = *reinterpret_cast<const float4*>(vec + q0 + j);
                const float4 d4 = *reinterpret_cast<const float4*>(vec + BQ + q0 + j);
                const float nlv[4] = {nl4.x, nl4.y, nl4.z, nl4.w};
                const float dv[4] = {d4.x, d4.y, d4.z, d4.w};
                float p[4], d[4];
#pragma unroll
                for (int t = 0; t < 4; t += 2) {  // two queries per paired fp32 instruction
                  float x0, x1;
                  f2_unpack(fma2(f2_pack(__uint_as_float(rs[bb][j + t]), __uint_as_float(rs[bb][j + t + 1])), sc2,
                                 f2_pack(nlv[t], nlv[t + 1])), x0, x1);
                  p[t] = fast_exp2(x0);
                  p[t + 1] = fast_exp2(x1);
                  if (DIAG && r_local > moff + q0 + j + t) p[t] = 0.f;
                  if (DIAG && r_local > moff + q0 + j + t + 1) p[t + 1] = 0.f;
                  f2_unpack(mul2(f2_pack(p[t], p[t + 1]),
                                 sub2(f2_pack(__uint_as_float(rd[bb][j + t]), __uint_as_float(rd[bb][j + t + 1])),
                                      f2_pack(dv[t], dv[t + 1]))),
                            d[t], d[t + 1]);
                }
                pp[g * 8 + (j >> 1)] = pack_bf16(p[0], p[1]);
                pp[g * 8 + (j >> 1) + 1] = pack_bf16(p[2], p[3]);
                dd[g * 8 + (j >> 1)] = pack_bf16(d[0], d[1]);
                dd[g * 8 + (j >> 1) + 1] = pack_bf16(d[2], d[3]);
              }
              if (g + 1 < NG) tmem_ld_wait();
            }
            tc_fence_before();
            mbar_arrive(sd_used);
            if (n > 0) {
              ok = bounded_wait_warp(mm_done, (n - 1) & 1, DEV_TIMEOUT_ATTN);
              if (!ok) return;
              tc_fence_after();
            }
            tmem_st16(t_lane + C_P + (uint32_t)(cs * (QCOLS / 2)), pp);
            // dS^T row segment -> shared memory ([key][64 queries], 128-byte swizzle)
            uint8_t* rowp = sds + r_local * 128;
            const int t0 = cs * (QCOLS / 8);
#pragma unroll
            for (int t = 0; t < QCOLS / 8; ++t)
              *reinterpret_cast<uint4*>(rowp + (((t0 + t) ^ (r_local & 7)) * 16)) =
                  make_uint4(dd[t * 4], dd[t * 4 + 1], dd[t * 4 + 2], dd[t * 4 + 3]);
          };
          if (i < 2) chunks(std::integral_constant<bool, true>{});
          else chunks(std::integral_constant<bool, false>{});
          if (ok) {
            tmem_st_wait();
            tc_fence_before();
            fence_async_smem();
            mbar_arrive(ds_ready);
          }
        }
        if (ok && n > 0) {
          if (i > 0) {
            uint32_t dq[32];
            dq_load(dq);
            dq_store(dq, prev_y);
          } else {
            unit_out(pu, prev_y);
          }
        }
        prev_y = (int)((size_t)un.bh * S + (size_t)(2 * un.kb + i) * BQ);
      }
      pu = un;
      if (!ok) break;
    }
    if (n > 0 && ok && bounded_wait_warp(mm_done, (n - 1) & 1, DEV_TIMEOUT_ATTN)) unit_out(pu, prev_y);
    if (lane == 0) bulk_wait0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
}  // namespace bwd128
}  // namespace fatc

namespace {
// Views of Q, K and V (or of dK and dV): `ld` elements between consecutive tokens.  The model's packed
// [T, 3E] activation is three views of one buffer (ld = 3E); the reference-style API passes three
// separate [T, E] tensors (ld = E).  Boxes are 64 head-dim columns by `box_rows` tokens.
bool bf16_view_map(CUtensorMap* m, const __nv_bfloat16* p, int E, int T, int ld, int box_cols, int box_rows,
                   int swizzle = 128) {
  return make_tma_map(m, p, false, (uint64_t)E, (uint64_t)T, box_cols, box_rows, swizzle, (uint64_t)ld);
}
bool aligned16(std::initializer_list<const void*> ps) {
  uintptr_t a = 0;
  for (const void* p : ps) a |= reinterpret_cast<uintptr_t>(p);
  return (a & 15) == 0;
}
}  // namespace

// Returns true if a tcgen05 kernel handled the call (head dim 64 or 128, S a multiple of 128, 16-byte
// aligned views with a row stride `ld` that is a multiple of 8).
bool fa_fwd_tc_launch3(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, int ld,
                       __nv_bfloat16* out, float* lse, int B, int S, int H, int Dh, cudaStream_t st, zl_status* status) {
  if ((Dh != 64 && Dh != 128) || S % fatc::BQ != 0 || ld % 8 != 0 || !aligned16({q, k, v})) return false;
  CUtensorMap tq, tk, tv;
  const int E = H * Dh, T = B * S;
  if (!bf16_view_map(&tq, q, E, T, ld, 64, 128) || !bf16_view_map(&tk, k, E, T, ld, 64, 128) ||
      !bf16_view_map(&tv, v, E, T, ld, 64, 128)) {
    *status = set_error(ZL_ECUDA, "attention: cuTensorMapEncodeTiled failed");
    return true;
  }
  const float scale_log2 = (1.0f / sqrtf((float)Dh)) * 1.4426950408889634f;
  // Persistent two-tile kernel when the sequence holds whole tile pairs and there are enough pairs
  // to give every SM one; ZL_ATTN_FWD_PP=0/1 forces either kernel (pairs permitting).
  const int nunits = S % (2 * fatc::BQ) == 0 ? B * H * (S / (2 * fatc::BQ)) : 0;
  const int sms = sm_count_current();
  const char* force = getenv("ZL_ATTN_FWD_PP");
  const bool pp = nunits > 0 && (force ? force[0] == '1' : nunits >= sms);
  if (pp) {
    const int grid = nunits < sms ? nunits : sms;
    auto launch_pp = [&](auto kern, int smem) {
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      kern<<<grid, fatc::THREADS_PP, smem, st>>>(tq, tk, tv, out, lse, S, H, nunits, scale_log2);
    };
    if (Dh == 64) launch_pp(fatc::fa_fwd_pp_kernel<64>, fatc::FwdPP<64>::SMEM_TOTAL);
    else launch_pp(fatc::fa_fwd_pp_kernel<128>, fatc::FwdPP<128>::SMEM_TOTAL);
    *status = check_launch("fa_fwd_pp_kernel");
    return true;
  }
  const int grid = B * H * (S / fatc::BQ);
  auto launch = [&](auto kern, int smem) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    kern<<<grid, fatc::THREADS, smem, st>>>(tq, tk, tv, out, lse, S, H, scale_log2);
  };
  if (Dh == 64) launch(fatc::fa_fwd_tc_kernel<64>, fatc::Fwd<64>::SMEM_TOTAL);
  else launch(fatc::fa_fwd_tc_kernel<128>, fatc::Fwd<128>::SMEM_TOTAL);
  *status = check_launch("fa_fwd_tc_kernel");
  return true;
}
bool fa_fwd_tc_launch(const __nv_bfloat16* qkv, __nv_bfloat16* out, float* lse, int B, int S, int H, int Dh,
                      cudaStream_t st, zl_status* status) {
  const int E = H * Dh;
  return fa_fwd_tc_launch3(qkv, qkv + E, qkv + 2 * E, 3 * E, out, lse, B, S, H, Dh, st, status);
}

// Whether a tcgen05 backward takes this call: head_dim 64 or 128, S a multiple of 128, and 16-byte
// aligned TMA sources, dQ accumulator and gradient views.
bool fa_bwd_tc_supported3(const void* q, const void* k, const void* v, int ld_in, const void* d_o, const void* dq_acc,
                          const void* dk, const void* dv, int ld_out, int S, int Dh) {
  return (Dh == 64 || Dh == 128) && S % fatc::BQ == 0 && ld_in % 8 == 0 && ld_out % 8 == 0 &&
         aligned16({q, k, v, d_o, dq_acc, dk, dv});
}
bool fa_bwd_tc_supported(const void* qkv, const void* d_o, const void* dq_acc, const void* d_qkv, int S, int Dh) {
  return fa_bwd_tc_supported3(qkv, qkv, qkv, 8, d_o, dq_acc, d_qkv, d_qkv, 8, S, Dh);
}

// Head-dim-64 backward form: a dedicated TMEM-readout warpgroup (512 threads) unless
// ZL_ATTN_BWD_READOUT=0 selects the form whose softmax warps read dQ / dK / dV out themselves.
static bool attn_bwd_readout_warps() {
  const char* f = getenv("ZL_ATTN_BWD_READOUT");
  return f ? f[0] != '0' : true;
}

// Backward main pass.  Before it the caller's pre pass writes nl = -lse*log2(e) and D = rowsum(dO*O)
// ([B, H, S]) and zeroes dq_acc and the unit counter; after it the post pass turns dq_acc
// ([B, H, S, Dh] fp32) into dQ.  dK is multiplied by `dk_scale` (the softmax scale; 1 for the
// reference's unscaled gradient).
zl_status fa_bwd_tc_launch3(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, int ld_in,
                            const __nv_bfloat16* d_o, const float* nl, const float* Dsum, float* dq_acc,
                            __nv_bfloat16* dk, __nv_bfloat16* dv, int ld_out, const float* rope_cos,
                            const float* rope_sin, int* unit_ctr, int B, int S, int H, int Dh, float dk_scale,
                            cudaStream_t st) {
  if (!unit_ctr) return set_error(ZL_EINVAL, "attention bwd: null unit counter");
  CUtensorMap tq, tk, tv, tdo, tdq, tdk, tdv;
  const int E = H * Dh, T = B * S;
  const float scale = 1.0f / sqrtf((float)Dh);
  const int nunits = B * H * (S / fatc::BKV);
  const int sms = sm_count_current();
  const int grid = nunits < sms ? nunits : sms;
  // Units are taken one head at a time (heaviest key block first) when the fp32 dQ accumulator is
  // too large to stay in L2 while every head's units run together: measured at batch 8 x 16 heads x
  // 2048 x 128 (a 134 MB accumulator) 756 us against 948 us; at batch 16 x 8 heads x 2048 x 64 (67 MB)
  // the key-block-major order over all heads is faster (311 us against 327 us).
  const int hgroup = (double)B * H * S * Dh * 4.0 > 96e6 ? 1 : 0;
  if (Dh == 128) {
    namespace K = fatc::bwd128;
    // K / V: 128-row boxes; Q / dO: 64-row boxes (64 head dims per box); dK / dV out: [32][64] boxes
    if (!bf16_view_map(&tq, q, E, T, ld_in, 64, K::BQ) || !bf16_view_map(&tk, k, E, T, ld_in, 64, K::BKV) ||
        !bf16_view_map(&tv, v, E, T, ld_in, 64, K::BKV) || !bf16_view_map(&tdo, d_o, E, T, E, 64, K::BQ) ||
        !make_tma_map(&tdq, dq_acc, true, (uint64_t)Dh, (uint64_t)B * H * S, 32, 32) ||
        !bf16_view_map(&tdk, dk, E, T, ld_out, 64, 32) || !bf16_view_map(&tdv, dv, E, T, ld_out, 64, 32))
      return set_error(ZL_ECUDA, "attention bwd: cuTensorMapEncodeTiled failed");
    cudaFuncSetAttribute(K::fa_bwd_tc128_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, K::SMEM_TOTAL);
    K::fa_bwd_tc128_kernel<<<grid, K::THREADS, K::SMEM_TOTAL, st>>>(
        tq, tk, tv, tdo, tdq, tdk, tdv, nl, Dsum, rope_cos, rope_sin, unit_ctr, S, H, nunits, hgroup, dk_scale,
        scale * 1.4426950408889634f);
    return check_launch("fa_bwd_tc128_kernel");
  }
  if (!bf16_view_map(&tq, q, E, T, ld_in, 64, 128) || !bf16_view_map(&tk, k, E, T, ld_in, 64, 128) ||
      !bf16_view_map(&tv, v, E, T, ld_in, 64, 128) || !bf16_view_map(&tdo, d_o, E, T, E, 64, 128) ||
      !make_tma_map(&tdq, dq_acc, true, (uint64_t)Dh, (uint64_t)B * H * S, 32, 32) ||
      !bf16_view_map(&tdk, dk, E, T, ld_out, 32, 32, 64) || !bf16_view_map(&tdv, dv, E, T, ld_out, 32, 32, 64))
    return set_error(ZL_ECUDA, "attention bwd: cuTensorMapEncodeTiled failed");
  if (attn_bwd_readout_warps()) {
    cudaFuncSetAttribute(fatc::bwd::fa_bwd_tc_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         fatc::bwd::SMEM_TOTAL);
    fatc::bwd::fa_bwd_tc_kernel<true><<<grid, fatc::bwd::THREADS_BQ, fatc::bwd::SMEM_TOTAL, st>>>(
        tq, tk, tv, tdo, tdq, tdk, tdv, nl, Dsum, rope_cos, rope_sin, unit_ctr, S, H, nunits, hgroup, dk_scale,
        scale * 1.4426950408889634f);
  } else {
    cudaFuncSetAttribute(fatc::bwd::fa_bwd_tc_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         fatc::bwd::SMEM_TOTAL);
    fatc::bwd::fa_bwd_tc_kernel<false><<<grid, fatc::bwd::THREADS_B, fatc::bwd::SMEM_TOTAL, st>>>(
        tq, tk, tv, tdo, tdq, tdk, tdv, nl, Dsum, rope_cos, rope_sin, unit_ctr, S, H, nunits, hgroup, dk_scale,
        scale * 1.4426950408889634f);
  }
  return check_launch("fa_bwd_tc_kernel");
}
zl_status fa_bwd_tc_launch(const __nv_bfloat16* qkv, const __nv_bfloat16* d_o, const float* nl, const float* Dsum,
                           float* dq_acc, __nv_bfloat16* d_qkv, const float* rope_cos, const float* rope_sin,
                           int* unit_ctr, int B, int S, int H, int Dh, cudaStream_t st) {
  const int E = H * Dh;
  return fa_bwd_tc_launch3(qkv, qkv + E, qkv + 2 * E, 3 * E, d_o, nl, Dsum, dq_acc, d_qkv + E, d_qkv + 2 * E, 3 * E,
                           rope_cos, rope_sin, unit_ctr, B, S, H, Dh, 1.0f / sqrtf((float)Dh), st);
}

int attn_tc_dev_error_read_and_clear() {
  int v = 0;
  cudaMemcpyFromSymbol(&v, zl_dev_error, sizeof(int));
  if (v) {
    int z = 0;
    cudaMemcpyToSymbol(zl_dev_error, &z, sizeof(int));
  }
  return v;
}

}  // namespace zl

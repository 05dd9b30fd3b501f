// Persistent warp-specialised bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   D[M, N] (+)= A[M, K] * B[N, K]^T      fp32 accumulation in tensor memory
//
// A and B are each K-major (row-major, K contiguous) or MN-major (their M/N index contiguous),
// which covers Y = X W^T (K/K), dX = dY W (K/MN) and dW = dY^T X (MN/MN) without transposes.
// Up to four row groups share A and K but carry their own B / bias / width (the video and text
// weights of the per-modality projections run in one launch).
//
// CTA = 192 threads, one CTA per SM (persistent: each CTA, or CTA pair, walks tiles t, t + grid, ...),
// tiles of 128 x 256 x 64 with a 4-stage smem ring, or for large problems 256 x 256 per CTA pair
// (cta_group::2, 6 stages; see Cfg below).  Tile order: bands of N tiles (8 wide, 16 for wide
// shallow-K launches) with the M tile outer inside a band, so a band's B tiles stay in L2 while A
// streams past (tile_coords; band_n_for picks the width):
//   warp 0      TMA producer (one lane): A/B tiles -> smem, completion on `full[s]`
//   warp 1      MMA issuer (one lane): 4 x tcgen05.mma 128x256x16 per stage, commit -> `empty[s]`;
//               owns the TMEM allocation (2 accumulators x 256 fp32 columns = 512 columns)
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time, bias / GELU-tanh / dGELU / accumulate,
//               bf16 or fp32 stores; releases the accumulator through `tmem_empty[acc]`
// The epilogue of tile i overlaps the main loop of tile i+1 (double-buffered accumulators).
// Every barrier wait is bounded (4 s): on timeout the kernel records an error code in
// g_error_flag and unwinds, so a bad launch cannot hang the GPU.
#include <mutex>

#include "common.cuh"
#include "launchers.h"
#include "sm100.cuh"

namespace pan {
namespace gemm {
using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int kThreads = 192;
constexpr int kMaxGroups = 4;

// CG = 1: one CTA per 128 x 256 tile.  CG = 2: a (2,1,1) cluster per 256 x 256 tile; each CTA holds
// its 128 A rows and 128 of the 256 B rows, which cuts the L2 -> SMEM bytes per FLOP by a third.
// Epilogue staging: every epilogue warp owns two 4 KB slots; a slot holds one 32-row x 32-column
// block of one output (bf16 with a 64-byte swizzle, fp32 with a 128-byte swizzle) that a TMA bulk
// store writes out as whole 64/128-byte row segments.
constexpr int EPI_SLOT = 4096;
constexpr int EPI_BYTES = 4 * 2 * EPI_SLOT;

template <int CG, int NSTAGES = (CG == 1 ? 4 : 6)>
struct Cfg {
  static constexpr int TILE_M = BM * CG;
  static constexpr int B_ROWS = BN / CG;                // B rows held by one CTA
  static constexpr int A_STAGE = BM * BK * 2;           // 16 KB
  static constexpr int B_STAGE = B_ROWS * BK * 2;       // 32 KB (CG 1) or 16 KB (CG 2)
  static constexpr int STAGES = NSTAGES;
  static constexpr int SMEM_BYTES = STAGES * (A_STAGE + B_STAGE) + EPI_BYTES + 1024 /*align*/ + 256 /*barriers*/;
};

enum Epi : int { EPI_PLAIN = 0, EPI_GELU = 1, EPI_DGELU = 2 };

struct Params {
  int M, N, K;            // M: total rows of A (for OOB); N: max width; K: reduction length
  int a_mn, b_mn;         // operand majors (1 = MN-major)
  int n_groups;
  int row_begin[kMaxGroups], row_end[kMaxGroups], n_cols[kMaxGroups];
  int tile_prefix[kMaxGroups + 1];
  int m_tiles[kMaxGroups], n_tiles[kMaxGroups];
  int k_blocks[kMaxGroups];  // per-group reduction length (groups may read a prefix of A's columns)
  const __nv_bfloat16* bias[kMaxGroups];
  void* D;
  long long ldd;
  int d_fp32;
  __nv_bfloat16* aux;     // GELU: pre-activation out; DGELU: pre-activation in
  long long ldaux;
  __nv_bfloat16* aux2;    // DGELU: GELU(pre) out
  long long ldaux2;
  int epi;
  int probe;  // timing experiments only: bit 0 skips the epilogue stores, bit 1 re-reads k-block 0
  int reduce_add;  // D += acc through TMA reduce-add stores (no read of D by the kernel)
  int band_m;      // tile order: 0 = N bands of band_n tiles, > 0 = M bands of band_m tiles
  int band_n;      // width of an N band in tiles (band_m == 0)
  int accumulate;  // host-side only: folded into C = D, beta = 1
  // batched GEMMs: operand z-coordinate = batch index; D/C advance by their batch strides
  int batch;
  int tiles_per_batch;
  long long d_bstride;
  // epilogue: out = alpha * acc + beta * C (+ bias); C may alias D
  float alpha, beta;
  const void* C;
  long long ldc, c_bstride;
  int c_fp32;
};

struct TmapSet {
  CUtensorMap a;
  CUtensorMap b[kMaxGroups];
  // outputs, one map per row group clipped at that group's rows / columns
  CUtensorMap d[kMaxGroups];
  CUtensorMap aux[kMaxGroups];
  CUtensorMap aux2[kMaxGroups];
};

// Tile order (per row group).  band_m == 0: bands of up to band_n N-tiles, M-tile outer within a band
// (consecutive tiles share A; for deep K the ~74 concurrent tiles form a near-square block).
// band_m > 0: bands of band_m M-tiles, N-tile outer, M-tile inner: the band's A rows (sized on the
// host to stay L2-resident) are read from DRAM once, and each B tile once per band.
__device__ __forceinline__ void tile_coords(const Params& p, int t, int& g, int& mb, int& nb) {
  t = t % p.tiles_per_batch;
  g = 0;
  while (g + 1 < p.n_groups && t >= p.tile_prefix[g + 1]) ++g;
  const int local = t - p.tile_prefix[g];
  const int mt = p.m_tiles[g], nt = p.n_tiles[g];
  if (p.band_m > 0) {
    const int band = local / (p.band_m * nt);
    const int height = min(p.band_m, mt - band * p.band_m);
    const int idx = local - band * p.band_m * nt;
    nb = idx / height;
    mb = band * p.band_m + idx % height;
    return;
  }
  const int bw = p.band_n;
  const int band = local / (mt * bw);
  const int width = min(bw, nt - band * bw);
  const int idx = local - band * mt * bw;
  mb = idx / width;
  nb = band * bw + idx % width;
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  return 0.5f * x * (1.f + tanhf(k0 * (x + k1 * x * x * x)));
}

__device__ __forceinline__ float gelu_tanh_grad(float x) {
  const float k0 = 0.7978845608028654f, k1 = 0.044715f;
  const float t = tanhf(k0 * (x + k1 * x * x * x));
  return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k0 * (1.f + 3.f * k1 * x * x);
}

template <int CG, int NSTAGES>
__global__ void __launch_bounds__(kThreads, 1)
gemm_kernel(const __grid_constant__ Params p, const __grid_constant__ TmapSet maps) {
  using C = Cfg<CG, NSTAGES>;
  constexpr int STAGES = C::STAGES, A_STAGE = C::A_STAGE, B_STAGE = C::B_STAGE;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* smem_a = smem;
  uint8_t* smem_b = smem + STAGES * A_STAGE;
  uint8_t* smem_epi = smem_b + STAGES * B_STAGE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem_epi + EPI_BYTES);
  // bars: full[S], empty[S], tmem_full[2], tmem_empty[2]; then the TMEM base address
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * STAGES + 4);
  volatile int& s_abort = *reinterpret_cast<volatile int*>(bars + 2 * STAGES + 5);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_tiles = p.tile_prefix[p.n_groups] * p.batch;
  // CG 2: the pair works on one tile; `crank` selects this CTA's half, rank 0 issues the MMAs
  const int crank = CG == 2 ? (int)cluster_ctarank() : 0;
  const int tile0 = CG == 2 ? (int)cluster_id_x() : (int)blockIdx.x;
  const int tile_step = CG == 2 ? (int)nclusters_x() : (int)gridDim.x;

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto tfull_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + 2 + a); };

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4 * CG);  // one arrive per epilogue warp of every CTA of the pair
    }
    fence_barrier_init();
    prefetch_tmap(&maps.a);
    for (int g = 0; g < p.n_groups; ++g) prefetch_tmap(&maps.b[g]);
  }
  if (warp == 1) {
    if (CG == 2) {
      tmem_alloc_pair(smem_u32(tmem_slot), 512);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(smem_u32(tmem_slot), 512);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();  // peer barriers initialised and TMEM allocated before any remote use
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int t = tile0; t < total_tiles && !s_abort; t += tile_step) {
        int g, mb, nb;
        tile_coords(p, t, g, mb, nb);
        const int m0 = p.row_begin[g] + mb * C::TILE_M + crank * BM;
        const int n0 = nb * BN + crank * C::B_ROWS;
        const int z = t / p.tiles_per_batch;
        const int k_blocks = p.k_blocks[g];
        for (int kb = 0; kb < k_blocks && !s_abort; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, 11)) { s_abort = 1; break; }
          // CG 2: both CTAs' bytes complete on the leader's full barrier
          const uint32_t fb = CG == 2 ? mapa_shared(full_bar(stage), 0) : full_bar(stage);
          if (crank == 0) mbar_expect_tx(full_bar(stage), CG * (A_STAGE + B_STAGE));
          const uint32_t sa = smem_u32(smem_a + stage * A_STAGE);
          const uint32_t sb = smem_u32(smem_b + stage * B_STAGE);
          const int k0 = (p.probe & 2) ? 0 : kb * BK;
          auto load = [&](uint32_t dst, const CUtensorMap* m, int c0, int c1) {
            if (CG == 2) tma_load_3d_pair(dst, m, fb, c0, c1, z);
            else tma_load_3d(dst, m, fb, c0, c1, z);
          };
          if (!p.a_mn) {
            load(sa, &maps.a, k0, m0);
          } else {
            load(sa, &maps.a, m0, k0);
            load(sa + 8192, &maps.a, m0 + 64, k0);
          }
          if (!p.b_mn) {
            load(sb, &maps.b[g], k0, n0);
          } else {
#pragma unroll
            for (int j = 0; j < C::B_ROWS / 64; ++j) load(sb + j * 8192, &maps.b[g], n0 + 64 * j, k0);
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (pair leader)
    if (lane == 0 && crank == 0) {
      const uint32_t idesc = idesc_bf16_f32(C::TILE_M, BN, p.a_mn, p.b_mn);
      // K-major SW128: LBO unused (16 B), SBO = 8 rows * 128 B; K step of 16 = +32 B.
      // MN-major SW128: LBO = next 64-wide MN chunk (8 KB), SBO = next 8 k-rows (1 KB); K step = +2 KB.
      const uint32_t a_lbo = p.a_mn ? 8192 : 16, b_lbo = p.b_mn ? 8192 : 16;
      const uint32_t a_kstep = p.a_mn ? 2048 : 32, b_kstep = p.b_mn ? 2048 : 32;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int t = tile0; t < total_tiles && !s_abort; t += tile_step) {
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1, 12)) { s_abort = 1; break; }
        tc_fence_after();
        int g, mb, nb;
        tile_coords(p, t, g, mb, nb);
        const int k_blocks = p.k_blocks[g];
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, 13)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem_a + stage * A_STAGE);
          const uint32_t sb = smem_u32(smem_b + stage * B_STAGE);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(sa + kk * a_kstep, a_lbo, 1024);
            const uint64_t bd = smem_desc_sw128(sb + kk * b_kstep, b_lbo, 1024);
            if (CG == 2) mma_bf16_ss_pair(d_tmem, ad, bd, idesc, (kb | kk) != 0);
            else mma_bf16_ss(d_tmem, ad, bd, idesc, (kb | kk) != 0);
          }
          // frees the smem stage (in both CTAs of a pair) when these MMAs retire
          if (CG == 2) mma_commit_pair(empty_bar(stage), 0x3);
          else mma_commit(empty_bar(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) { s_abort = 1; break; }
        if (CG == 2) mma_commit_pair(tfull_bar(acc), 0x3);  // accumulator ready for both epilogues
        else mma_commit(tfull_bar(acc));
        if (++acc == 2) { acc = 0; acc_phase ^= 1; }
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint8_t* slots = smem_epi + q * 2 * EPI_SLOT;
    int n_used = 0;
    // next staging slot; the bulk store that last read it (two stores ago) must have finished reading
    auto acquire = [&]() -> uint8_t* {
      uint8_t* b = slots + (n_used & 1) * EPI_SLOT;
      if (n_used >= 2 && lane == 0) bulk_wait_read<1>();
      __syncwarp();
      ++n_used;
      return b;
    };
    // this lane's row of a 32 x 32 block: bf16 rows of 64 B (64-byte swizzle), fp32 rows of 128 B
    auto put_bf16 = [&](uint8_t* b, const float* v) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 w;
        w.x = pack_bf16(v[8 * j + 0], v[8 * j + 1]);
        w.y = pack_bf16(v[8 * j + 2], v[8 * j + 3]);
        w.z = pack_bf16(v[8 * j + 4], v[8 * j + 5]);
        w.w = pack_bf16(v[8 * j + 6], v[8 * j + 7]);
        *reinterpret_cast<uint4*>(b + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4)) = w;
      }
    };
    auto put_f32 = [&](uint8_t* b, const float* v) {
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<float4*>(b + lane * 128 + ((j ^ (lane & 7)) << 4)) =
            make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    };
    // Coalesced read of a 32-row x 32-column block (rows row0.., columns c0..) through a staging
    // slot: the warp loads whole 64 / 128-byte row segments, then each lane takes its own row.
    // Rows at or past `row_lim` and columns at or past `col_lim` read as zero.
    auto get_bf16 = [&](uint8_t* b, const __nv_bfloat16* src, long long ld, int row0_, int c0_, int row_lim,
                        int col_lim, float* v) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int r = k * 8 + (lane >> 2), part = lane & 3;
        const int rr = row0_ + r, cc = c0_ + part * 8;
        uint4 w = make_uint4(0u, 0u, 0u, 0u);
        if (rr < row_lim && cc < col_lim) w = *reinterpret_cast<const uint4*>(src + (size_t)rr * ld + cc);
        *reinterpret_cast<uint4*>(b + r * 64 + ((part ^ ((r >> 1) & 3)) << 4)) = w;
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 w = *reinterpret_cast<const uint4*>(b + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4));
        const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[e]));
          v[8 * j + 2 * e] = f.x;
          v[8 * j + 2 * e + 1] = f.y;
        }
      }
      __syncwarp();
    };
    auto get_f32 = [&](uint8_t* b, const float* src, long long ld, int row0_, int c0_, int row_lim, int col_lim,
                       float* v) {
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int r = k * 4 + (lane >> 3), part = lane & 7;
        const int rr = row0_ + r, cc = c0_ + part * 4;
        float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rr < row_lim && cc < col_lim) w = *reinterpret_cast<const float4*>(src + (size_t)rr * ld + cc);
        *reinterpret_cast<float4*>(b + r * 128 + ((part ^ (r & 7)) << 4)) = w;
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float4 w = *reinterpret_cast<const float4*>(b + lane * 128 + ((j ^ (lane & 7)) << 4));
        v[4 * j] = w.x;
        v[4 * j + 1] = w.y;
        v[4 * j + 2] = w.z;
        v[4 * j + 3] = w.w;
      }
      __syncwarp();
    };
    auto issue = [&](const CUtensorMap* m, uint8_t* b, int col, int row, int z, bool add = false) {
      fence_async_shared();
      __syncwarp();
      if (lane == 0) {
        if (add) tma_reduce_add_3d(m, smem_u32(b), col, row, z);
        else tma_store_3d(m, smem_u32(b), col, row, z);
        bulk_commit();
      }
    };
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = tile0; t < total_tiles && !s_abort; t += tile_step) {
      if (!mbar_wait(tfull_bar(acc), acc_phase, 14)) { s_abort = 1; break; }
      tc_fence_after();
      int g, mb, nb;
      tile_coords(p, t, g, mb, nb);
      const int zb = t / p.tiles_per_batch;
      const int row0 = p.row_begin[g] + mb * C::TILE_M + crank * BM + q * 32;  // first row of this warp
      const int row = row0 + lane;
      const bool row_ok = row < p.row_end[g];
      const int n_lim = p.n_cols[g];
      const __nv_bfloat16* bias = p.bias[g];
      const uint32_t t_row = tmem_base + acc * BN + ((uint32_t)(q * 32) << 16);
      for (int ch = 0; ch < BN / 32; ++ch) {
        const int c0 = nb * BN + ch * 32;
        uint32_t r[32];
        tmem_ld32(t_row + ch * 32, r);
        tmem_ld_wait();
        if (c0 >= n_lim || (p.probe & 1)) continue;
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = p.alpha * __uint_as_float(r[i]);
        if (p.C != nullptr) {
          float cv[32];
          uint8_t* sb = acquire();  // used as scratch, then released for the next output
          if (p.c_fp32)
            get_f32(sb, reinterpret_cast<const float*>(p.C) + zb * p.c_bstride, p.ldc, row0, c0, p.row_end[g], n_lim, cv);
          else
            get_bf16(sb, reinterpret_cast<const __nv_bfloat16*>(p.C) + zb * p.c_bstride, p.ldc, row0, c0, p.row_end[g],
                     n_lim, cv);
          --n_used;  // nothing was stored from this slot
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] += p.beta * cv[i];
        }
        if (bias != nullptr) {
#pragma unroll
          for (int v8 = 0; v8 < 4; ++v8) {
            const int c = c0 + v8 * 8;
            if (c >= n_lim) break;
            float b[8];
            load8(bias + c, b);
#pragma unroll
            for (int i = 0; i < 8; ++i) o[v8 * 8 + i] += b[i];
          }
        }
        if (p.epi == EPI_GELU) {
          uint8_t* sb = acquire();
          put_bf16(sb, o);  // pre-activation
          issue(&maps.aux[g], sb, c0, row0, zb);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = gelu_tanh(__bfloat162float(__float2bfloat16_rn(o[i])));
        } else if (p.epi == EPI_DGELU) {
          float pre[32];
          uint8_t* sb = acquire();
          get_bf16(sb, p.aux, p.ldaux, row0, c0, p.row_end[g], n_lim, pre);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= gelu_tanh_grad(pre[i]);
#pragma unroll
          for (int i = 0; i < 32; ++i) pre[i] = gelu_tanh(pre[i]);
          put_bf16(sb, pre);  // post-activation (same slot)
          issue(&maps.aux2[g], sb, c0, row0, zb);
        }
        uint8_t* sb = acquire();
        if (p.d_fp32) put_f32(sb, o);
        else put_bf16(sb, o);
        issue(&maps.d[g], sb, c0, row0, zb, p.reduce_add != 0);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        // the leader's MMA warp reuses the accumulator once every epilogue warp of the pair is done
        if (CG == 2) mbar_arrive_cluster(mapa_shared(tempty_bar(acc), 0));
        else mbar_arrive(tempty_bar(acc));
      }
      if (++acc == 2) { acc = 0; acc_phase ^= 1; }
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (CG == 2) cluster_sync();  // the peer's MMAs / arrivals target this CTA until both are done
  if (warp == 1) {
    tc_fence_after();
    if (CG == 2) tmem_dealloc_pair(tmem_base, 512);
    else tmem_dealloc(tmem_base, 512);
  }
}

// ---------------------------------------------------------------------------------- host side

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 3-D tensor map over `batch` row-major [rows, cols] matrices (row stride `ld`, batch stride `bstride`
// elements), box [1, box_rows, box_cols].  Operand maps use bf16 with a 128-byte swizzle (box_cols * 2
// == 128); output maps use bf16 / fp32 with the swizzle matching their 64 / 128-byte box rows.
const char* make_map(CUtensorMap* m, const void* base, long long rows, long long cols, long long ld, int box_rows,
                     int box_cols, int batch = 1, long long bstride = 0,
                     CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, int esize = 2,
                     CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_128B) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) return "TMA base must be 16-byte aligned";
  if ((ld * esize) % 16 != 0) return "TMA row stride must be a multiple of 16 bytes";
  if (batch > 1 && (bstride * esize) % 16 != 0) return "TMA batch stride must be a multiple of 16 bytes";
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return "cuTensorMapEncodeTiled is unavailable";
  if (rows < 1) rows = 1;
  if (batch <= 1) bstride = ld * rows;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)(batch < 1 ? 1 : batch)};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * esize), (cuuint64_t)(bstride * esize)};
  cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(m, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? nullptr : "cuTensorMapEncodeTiled failed";
}

// Output map of one row group: clipped at the group's last row and column, 32 x 32 boxes.
const char* make_out_map(CUtensorMap* m, const void* base, int row_end, int n, long long ld, bool fp32, int batch,
                         long long bstride) {
  return make_map(m, base, row_end, n, ld, 32, 32, batch, bstride,
                  fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, fp32 ? 4 : 2,
                  fp32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

int g_forced_cta_group = 0;  // 0: choose per launch; 1 / 2: force (tests, A/B timing)
int g_pair_stages = 6;       // smem stages of the CTA-pair kernel (4 or 6)
int g_probe = 0;             // Params::probe of every launch (timing experiments)
// Tile order: A rows of one M band up to g_band_mb MB (0 = always N bands).  M bands are used when a
// 128/256-row A tile is at most 4 MB (K <= 8192): then the band stays in L2 while B streams past.
int g_band_mb = 0;
// N-band width in tiles (0: by shape).  A is re-read once per band, and the band's B tiles stay in
// L2 while the M tiles stream past, so wider bands trade L2 room for fewer A passes.  Measured on
// the 29B shapes (94,960 rows): 16-tile bands cut the FFN up-projection and its input gradient
// (N = 32768, K = 4096) by 6-8 % and let the clock settle higher under the power cap (less DRAM
// traffic); the QKV projection (N = 12288) ran 12 % slower with them and the deep-K shapes
// (K >= 32768) were flat, so those keep 8.
int g_band_n = 0;
inline int band_n_for(int K, int max_n_tiles) { return (K <= 8192 && max_n_tiles >= 64) ? 16 : 8; }

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

}  // namespace gemm

const char* launch_gemm(const GemmArgs& a, cudaStream_t stream) {
  using namespace gemm;
  const int G = a.n_groups;
  if (G < 1 || G > kMaxGroups) return "gemm: 1..4 groups";
  if (a.lda % 8 != 0) return "gemm: A row stride must be a multiple of 8 elements";
  if (a.ldd % 8 != 0 && !a.d_fp32) return "gemm: D row stride must be a multiple of 8 elements";
  if (a.d_fp32 && a.ldd % 4 != 0) return "gemm: fp32 D row stride must be a multiple of 4 elements";
  Params p{};
  p.M = a.M;
  p.K = a.K;
  p.a_mn = a.a_mn;
  p.b_mn = a.b_mn;
  p.n_groups = G;
  p.D = a.D;
  p.ldd = a.ldd;
  p.d_fp32 = a.d_fp32;
  p.epi = a.epi;
  p.accumulate = a.accumulate;
  p.aux = reinterpret_cast<__nv_bfloat16*>(a.aux);
  p.ldaux = a.ldaux;
  p.aux2 = reinterpret_cast<__nv_bfloat16*>(a.aux2);
  p.ldaux2 = a.ldaux2;
  p.batch = a.batch < 1 ? 1 : a.batch;
  p.d_bstride = a.d_bstride;
  p.alpha = a.alpha;
  p.beta = a.beta;
  p.C = a.C;
  p.ldc = a.ldc;
  p.c_bstride = a.c_bstride;
  p.c_fp32 = a.c_fp32;
  if (a.accumulate) {
    if (a.C == nullptr && a.epi == EPI_PLAIN && a.d_fp32) {
      // D += alpha * acc (+ bias): the L2 adds through TMA reduce-add stores; D is never read
      p.reduce_add = 1;
    } else {  // D += acc  ==  C = D, beta = 1
      p.C = a.D;
      p.ldc = a.ldd;
      p.c_bstride = a.d_bstride;
      p.c_fp32 = a.d_fp32;
      p.beta = 1.f;
    }
  }
  if (p.C != nullptr && (p.ldc % 8 != 0 && !p.c_fp32)) return "gemm: C row stride must be a multiple of 8";
  // CTA pairs for large single-batch GEMMs whose row groups fill 256-row tiles; the batched
  // 128-row Gram products of Muon and small problems keep one CTA per tile.
  int min_rows = 1 << 30;
  long long pair_tiles = 0;
  for (int g = 0; g < G; ++g) {
    const int rows = a.groups[g].row_end > a.groups[g].row_begin ? a.groups[g].row_end - a.groups[g].row_begin : 0;
    if (rows > 0) min_rows = rows < min_rows ? rows : min_rows;
    pair_tiles += (long long)((rows + 255) / 256) * ((a.groups[g].n + BN - 1) / BN);
  }
  int cg = (p.batch == 1 && min_rows >= 256 && pair_tiles >= 16) ? 2 : 1;
  const int forced = g_forced_cta_group;
  if (forced == 1 || (forced == 2 && p.batch == 1)) cg = forced;
  const int tile_m = BM * cg;
  const int b_rows = BN / cg;
  TmapSet maps;
  const char* err = !a.a_mn ? make_map(&maps.a, a.A, a.M, a.K, a.lda, BM, BK, p.batch, a.a_bstride)
                            : make_map(&maps.a, a.A, a.K, a.M, a.lda, BK, 64, p.batch, a.a_bstride);
  if (err) return err;
  int tiles = 0;
  p.tile_prefix[0] = 0;
  for (int g = 0; g < G; ++g) {
    const GemmGroup& gr = a.groups[g];
    if (gr.k > a.K) return "gemm: group K must be <= K";
    if (gr.ldb % 8 != 0) return "gemm: B row stride must be a multiple of 8 elements";
    if (gr.n % 8 != 0) return "gemm: N must be a multiple of 8";
    err = !a.b_mn ? make_map(&maps.b[g], gr.B, gr.n, gr.k, gr.ldb, b_rows, BK, p.batch, a.b_bstride)
                  : make_map(&maps.b[g], gr.B, gr.k, gr.n, gr.ldb, BK, 64, p.batch, a.b_bstride);
    if (err) return err;
    err = make_out_map(&maps.d[g], a.D, gr.row_end, gr.n, a.ldd, a.d_fp32, p.batch, a.d_bstride);
    if (err) return err;
    if (a.epi == EPI_GELU) err = make_out_map(&maps.aux[g], a.aux, gr.row_end, gr.n, a.ldaux, false, 1, 0);
    else maps.aux[g] = maps.d[g];
    if (err) return err;
    if (a.epi == EPI_DGELU) err = make_out_map(&maps.aux2[g], a.aux2, gr.row_end, gr.n, a.ldaux2, false, 1, 0);
    else maps.aux2[g] = maps.d[g];
    if (err) return err;
    p.row_begin[g] = gr.row_begin;
    p.row_end[g] = gr.row_end;
    p.n_cols[g] = gr.n;
    p.k_blocks[g] = (gr.k + BK - 1) / BK;
    p.bias[g] = reinterpret_cast<const __nv_bfloat16*>(gr.bias);
    const int rows = gr.row_end > gr.row_begin ? gr.row_end - gr.row_begin : 0;
    p.m_tiles[g] = (rows + tile_m - 1) / tile_m;
    p.n_tiles[g] = (gr.n + BN - 1) / BN;
    tiles += p.m_tiles[g] * p.n_tiles[g];
    p.tile_prefix[g + 1] = tiles;
  }
  for (int g = G; g < kMaxGroups; ++g) {
    maps.b[g] = maps.b[0];
    maps.d[g] = maps.d[0];
    maps.aux[g] = maps.aux[0];
    maps.aux2[g] = maps.aux2[0];
  }
  p.tiles_per_batch = tiles;
  p.band_m = 0;
  int max_nt = 0;
  for (int g = 0; g < G; ++g) max_nt = p.n_tiles[g] > max_nt ? p.n_tiles[g] : max_nt;
  p.band_n = g_band_n > 0 ? g_band_n : band_n_for(a.K, max_nt);
  const long long a_tile_bytes = (long long)tile_m * a.K * 2;
  if (g_band_mb > 0 && a_tile_bytes <= (4ll << 20)) {
    const long long band = ((long long)g_band_mb << 20) / a_tile_bytes;
    p.band_m = (int)(band < 1 ? 1 : band);
  }
  tiles *= p.batch;
  if (tiles == 0) return nullptr;
  p.probe = g_probe;
  if (cg == 1) {
    static bool attr1 = false;
    if (!attr1) {
      if (cudaFuncSetAttribute(gemm_kernel<1, 4>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               Cfg<1, 4>::SMEM_BYTES) != cudaSuccess)
        return "gemm: cannot set the dynamic shared memory size";
      attr1 = true;
    }
    const int grid = tiles < num_sms() ? tiles : num_sms();
    gemm_kernel<1, 4><<<grid, kThreads, Cfg<1, 4>::SMEM_BYTES, stream>>>(p, maps);
  } else {
    const int clusters = tiles < num_sms() / 2 ? tiles : num_sms() / 2;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    switch (g_pair_stages) {
#define PAN_PAIR_LAUNCH(S)                                                                                         \
  case S: {                                                                                                      \
    static bool set = false;                                                                                     \
    if (!set) {                                                                                                  \
      if (cudaFuncSetAttribute(gemm_kernel<2, S>, cudaFuncAttributeMaxDynamicSharedMemorySize,                   \
                               Cfg<2, S>::SMEM_BYTES) != cudaSuccess)                                            \
        return "gemm: cannot set the dynamic shared memory size";                                                \
      set = true;                                                                                                \
    }                                                                                                            \
    cfg.dynamicSmemBytes = Cfg<2, S>::SMEM_BYTES;                                                                \
    e = cudaLaunchKernelEx(&cfg, gemm_kernel<2, S>, p, maps);                                                    \
    break;                                                                                                       \
  }
      PAN_PAIR_LAUNCH(4)
      default:
      PAN_PAIR_LAUNCH(6)
#undef PAN_PAIR_LAUNCH
    }
    if (e != cudaSuccess) return "gemm: pair launch failed";
  }
  return cudaGetLastError() == cudaSuccess ? nullptr : "gemm: launch failed";
}

void gemm_force_cta_group(int cg) { gemm::g_forced_cta_group = (cg == 1 || cg == 2) ? cg : 0; }
void gemm_tuning(int pair_stages, int probe, int band_mb, int band_n) {
  gemm::g_pair_stages = pair_stages == 4 ? 4 : 6;
  gemm::g_probe = probe;
  gemm::g_band_mb = band_mb < 0 ? 0 : band_mb;
  gemm::g_band_n = band_n < 0 ? 0 : band_n;
}

int gemm_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, sm100::g_error_flag, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(sm100::g_error_flag, &z, sizeof(int));
  }
  return v;
}

}  // namespace pan

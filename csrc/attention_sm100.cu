// Variable-length non-causal attention for sm_100a (tcgen05 + TMEM + TMA), head_dim 128.
// Replaces the reference's FlashAttention-4 varlen calls (pan/utils/flash_attention.py:18-86).
//
// Forward (one CTA = one head x two 128-row query tiles "A" and "B" of one segment; 10 warps):
//   warp 0       TMA: Q_A, Q_B once; then K_j, V_j through a 5-slot smem ring
//   warp 1       MMA (one lane): S_X = Q_X K_j^T into TMEM; O_X += P_X V_j with P_X read from TMEM
//                (bf16, written over the first 64 columns of S_X); the next S_X is issued right
//                behind PV_X (one thread's MMAs execute in order)
//   warps 2..5   softmax of tile A (one TMEM lane = one query row per thread)
//   warps 6..9   softmax of tile B
// The two tiles ping-pong: while one softmax group works, the tensor core runs the other tile's
// GEMMs.  Online softmax in the exp2 domain with lazy rescaling: O and l are rescaled only when
// the running max grows by more than 8 (a factor of 256), so most iterations leave O in TMEM
// untouched.  Outputs O (bf16, [L, H, D]) and the natural-log LSE ([H, L] fp32).
//
// Backward is one fused pass, key tiles outer (attn_bwd_fused_kernel): per 128-query tile S^T and
// dP^T on the tensor core, P^T / dS^T by the elementwise warps (P recomputed from the saved LSE),
// dV += P^T dO and dK += dS^T Q with P^T / dS^T as TMEM operands, dQ^T = K^T dS^T drained by four
// warps into an fp32 accumulator through TMA reduce-add stores, which a last kernel scales to bf16.
//
// Smem tiles are 128 rows x 64 columns bf16 with the 128-byte swizzle, two per 128-wide operand.
// The same bytes serve as a K-major operand (rows = M/N, e.g. K for S = Q K^T) or an MN-major one
// (rows = K, e.g. V for O += P V).  Every barrier wait is bounded (no hangs, error flag instead).
#include "common.cuh"
#include "launchers.h"
#include "sm100.cuh"

namespace pan {
namespace attn {
using namespace sm100;

constexpr int D = 128;
constexpr int BT = 128;                    // rows per tile (queries or keys)
constexpr int TILE_BYTES = BT * D * 2;     // 32 KB (two 16 KB swizzled halves)
constexpr int HALF_BYTES = TILE_BYTES / 2;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

struct WorkItem {
  int seg_start;   // first row of the segment
  int seg_len;     // rows of the segment
  int tile_start;  // first row (relative to seg_start) of this CTA's outer tile(s)
  int pad;
};

// Token-sharded destination of a Ulysses context-parallel group (the reverse all-to-all folded
// into a kernel's stores).  Attention runs on the FULL sequence for heads [head_base, head_base +
// H); global row g belongs to cp-rank g % cp at its local row g / cp, whose [rows, H_total, D]
// buffer starts at base[g % cp] (an address in that rank's memory, mapped over NVLink).  Only
// plain vector stores go through these addresses.
struct PeerRows {
  const uint64_t* base;  // nullptr: off
  int cp, head_base, H_total;
};

__device__ __forceinline__ __nv_bfloat16* peer_row(const PeerRows& pr, int g, int h) {
  return reinterpret_cast<__nv_bfloat16*>(pr.base[g % pr.cp]) +
         ((size_t)(g / pr.cp) * pr.H_total + pr.head_base + h) * D;
}

// K-major SW128 descriptor of a [128 rows, 128 cols] operand at k-step kk (16 columns per step).
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t base, int kk) {
  return smem_desc_sw128(base + (kk >> 2) * HALF_BYTES + (kk & 3) * 32, 16, 1024);
}
// MN-major SW128 descriptor: rows are the reduction dim; k-step of 16 rows = 2 KB; the two
// 64-wide column halves are 16 KB apart.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t base, int kk) {
  return smem_desc_sw128(base + kk * 2048, HALF_BYTES, 1024);
}

// Write 32 consecutive bf16 values (16 packed words) of row `r`, columns [c0, c0+32) into a
// swizzled [128, 128] K-major smem operand.
__device__ __forceinline__ void store_row32_swizzled(uint8_t* tile, int r, int c0, const uint32_t (&w)[16]) {
  uint8_t* half = tile + (c0 >> 6) * HALF_BYTES + r * 128;
  const int u0 = (c0 & 63) >> 3;  // 16-byte unit within the 128-byte row
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int u = (u0 + j) ^ (r & 7);
    *reinterpret_cast<uint4*>(half + u * 16) = make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
  }
}

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 2^x on the SFU (PTX ex2.approx.ftz.f32, ~2 ulp); softmax probabilities are rounded to bf16 anyway.
// Packed fp32 pair arithmetic (one instruction for two lanes' worth of FMA / add) and a 3-input
// max: the forward softmax is bound by instruction issue, not by the MUFU exponentials.
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 ra, rb, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// ============================================================================ forward
constexpr int FWD_THREADS = 320;
constexpr int FWD_RING = 5;  // K/V tiles in flight (P lives in TMEM, so the smem goes to the ring)
constexpr int FWD_SMEM = 2 * TILE_BYTES /*Q*/ + FWD_RING * TILE_BYTES + 1024 + 256;

// INORDER: the next score GEMM of a tile is issued right after that tile's PV GEMM.  tcgen05.mma
// instructions of one thread execute in issue order, so S(j+1) cannot overwrite the P(j) columns
// before PV(j) has read them and no completion wait is needed between them (measured: ~6 % less
// time per SM clock than awaiting PV's completion first, which the other instance does).
template <bool INORDER>
__global__ void __launch_bounds__(FWD_THREADS, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                const __grid_constant__ CUtensorMap vmap, const WorkItem* __restrict__ items, int L, int H,
                float scale_log2, __nv_bfloat16* __restrict__ out, float* __restrict__ lse, const PeerRows o_peer) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                 // 2 tiles
  uint8_t* sKV = sQ + 2 * TILE_BYTES;                 // FWD_RING tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + FWD_RING * TILE_BYTES);
  // bars: q_full, kv_full[R], kv_empty[R], s_full[2], p_ready[2], pv_done[2]
  constexpr int RB = 1 + 2 * FWD_RING;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + RB + 6);
  volatile int& s_abort = *reinterpret_cast<volatile int*>(bars + RB + 7);

  const WorkItem it = items[blockIdx.x];
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kv = (it.seg_len + BT - 1) / BT;

  const uint32_t q_full = smem_u32(bars + 0);
  auto kv_full = [&](int s) { return smem_u32(bars + 1 + s); };
  auto kv_empty = [&](int s) { return smem_u32(bars + 1 + FWD_RING + s); };
  auto s_full = [&](int x) { return smem_u32(bars + RB + x); };
  auto p_ready = [&](int x) { return smem_u32(bars + RB + 2 + x); };
  auto pv_done = [&](int x) { return smem_u32(bars + RB + 4 + x); };

  if (threadIdx.x == 0) {
    s_abort = 0;
    mbar_init(q_full, 1);
    for (int s = 0; s < FWD_RING; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(s_full(x), 1);
      mbar_init(p_ready(x), 4);
      mbar_init(pv_done(x), 1);
    }
    fence_barrier_init();
    prefetch_tmap(&qmap);
    prefetch_tmap(&kmap);
    prefetch_tmap(&vmap);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;  // S_A 0, S_B 128, O_A 256, O_B 384

  const int col = h * D;
  if (warp == 0) {
    if (lane == 0) {
      const int q0 = it.seg_start + it.tile_start;
      mbar_expect_tx(q_full, 2 * TILE_BYTES);
      for (int x = 0; x < 2; ++x) {
        const uint32_t dst = smem_u32(sQ + x * TILE_BYTES);
        tma_load_2d(dst, &qmap, q_full, col, q0 + x * BT);
        tma_load_2d(dst + HALF_BYTES, &qmap, q_full, col + 64, q0 + x * BT);
      }
      int n = 0;
      for (int j = 0; j < n_kv && !s_abort; ++j) {
        for (int w = 0; w < 2; ++w, ++n) {  // K_j then V_j
          const int slot = n % FWD_RING;
          const uint32_t ph = (n / FWD_RING) & 1;
          if (!mbar_wait(kv_empty(slot), ph ^ 1, 21)) { s_abort = 1; break; }
          const uint32_t fb = kv_full(slot);
          mbar_expect_tx(fb, TILE_BYTES);
          const uint32_t dst = smem_u32(sKV + slot * TILE_BYTES);
          const CUtensorMap* m = w == 0 ? &kmap : &vmap;
          const int row = it.seg_start + j * BT;
          tma_load_2d(dst, m, fb, col, row);
          tma_load_2d(dst + HALF_BYTES, m, fb, col + 64, row);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16_f32(128, 128, 0, 0);   // S = Q K^T
      const uint32_t id_pv = idesc_bf16_f32(128, 128, 0, 1);  // O += P V  (V is MN-major)
      bool ok = mbar_wait(q_full, 0, 22);
      tc_fence_after();
      auto wait_slot = [&](int n) {
        if (!ok) return 0u;
        const int slot = n % FWD_RING;
        ok = mbar_wait(kv_full(slot), (n / FWD_RING) & 1, 23);
        tc_fence_after();
        return smem_u32(sKV + slot * TILE_BYTES);
      };
      auto issue_s = [&](int x, uint32_t kb) {
        const uint32_t qb = smem_u32(sQ + x * TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma_bf16_ss(tmem + x * 128, desc_kmajor(qb, kk), desc_kmajor(kb, kk), id_s, kk > 0);
        mma_commit(s_full(x));
      };
      // O_x += P_x V_j with P_x (bf16, written over the first 64 columns of S_x) as the A operand
      auto issue_pv = [&](int x, uint32_t vb, bool acc) {
#pragma unroll
        for (int kk = 0; kk < BT / 16; ++kk)
          mma_bf16_ts(tmem + 256 + x * 128, tmem + x * 128 + kk * 8, desc_mnmajor(vb, kk), id_pv, acc || kk > 0);
        mma_commit(pv_done(x));
      };
      // S_x(j+1) overwrites the columns PV_x(j) reads P_x(j) from.  INORDER relies on the in-order
      // execution of one thread's MMAs; otherwise PV_x(j)'s completion is awaited first.
      auto next_s = [&](int x, uint32_t kb, int j) {
        if (!INORDER) {
          if (!(ok = mbar_wait(pv_done(x), j & 1, 29 + x))) return;
          tc_fence_after();
        }
        issue_s(x, kb);
      };
      // prologue: S_A(0), S_B(0)
      uint32_t kb = wait_slot(0);
      if (ok) {
        issue_s(0, kb);
        issue_s(1, kb);
        mma_commit(kv_empty(0));
      }
      for (int j = 0; j < n_kv && ok; ++j) {
        const int nv = 2 * j + 1, nk = 2 * j + 2;
        const uint32_t vb = wait_slot(nv);
        if (!ok) break;
        if (!(ok = mbar_wait(p_ready(0), j & 1, 24))) break;
        tc_fence_after();
        issue_pv(0, vb, j > 0);
        uint32_t kb2 = 0;
        if (j + 1 < n_kv) {
          kb2 = wait_slot(nk);
          if (!ok) break;
          next_s(0, kb2, j);
          if (!ok) break;
        }
        if (!(ok = mbar_wait(p_ready(1), j & 1, 25))) break;
        tc_fence_after();
        issue_pv(1, vb, j > 0);
        mma_commit(kv_empty(nv % FWD_RING));
        if (j + 1 < n_kv) {
          next_s(1, kb2, j);
          if (!ok) break;
          mma_commit(kv_empty(nk % FWD_RING));
        }
      }
      if (!ok) s_abort = 1;
    }
  } else {
    // ------------------------------------------------------------ softmax groups
    const int x = (warp - 2) >> 2;           // 0 = tile A, 1 = tile B
    const int quarter = warp & 3;            // TMEM lane quarter of this warp
    const int row = quarter * 32 + lane;     // query row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem + x * 128 + lane_off;
    const uint32_t tO = tmem + 256 + x * 128 + lane_off;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    // O and l are rescaled only when the running maximum grows by more than 8 (a factor of 256);
    // PV_x(j-1) must be complete before O is read
    auto maybe_rescale = [&](int j, float m_new) -> bool {
      const bool grow = m_new > m_used + 8.f;
      if (j > 0) {
        if (!mbar_wait(pv_done(x), (j - 1) & 1, 27)) return false;
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
          const float alpha = grow ? fast_exp2(m_used - m_new) : 1.f;  // m_used finite here (j > 0)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t o[32];
            tmem_ld32(tO + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(tO + c * 32, o);
          }
          tmem_st_wait();
          l *= alpha;
        }
      }
      if (grow) m_used = m_new;
      return true;
    };
    // exponentiate one 32-column chunk of scores into 16 packed bf16 P words; masked columns -> 0
    auto exp_chunk = [&](const uint32_t (&r)[32], int c0, int valid, uint32_t (&w)[16], float& l0, float& l1) {
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        float x0, x1;
        ffma2(x0, x1, __uint_as_float(r[i]), __uint_as_float(r[i + 1]), scale_log2, scale_log2, -m_used, -m_used);
        float p0 = fast_exp2(x0);
        float p1 = fast_exp2(x1);
        if (valid < BT) {
          p0 = c0 + i < valid ? p0 : 0.f;
          p1 = c0 + i + 1 < valid ? p1 : 0.f;
        }
        fadd2(l0, l1, l0, l1, p0, p1);
        w[i >> 1] = pack_bf16(p0, p1);
      }
    };
    for (int j = 0; j < n_kv; ++j) {
      if (ok) {
        ok = mbar_wait(s_full(x), j & 1, 26);
        tc_fence_after();
      }
      const int valid = min(BT, it.seg_len - j * BT);
      float l0 = 0.f, l1 = 0.f;
      // two TMEM passes (max, then exp), two 32-column chunks per TMEM wait (10 warps cap registers
      // at 168 per thread, so 64 scores are live at a time)
      float mx0 = -INFINITY, mx1 = -INFINITY;
      auto max_chunk = [&](const uint32_t (&r)[32], int c0) {
        if (valid == BT) {
#pragma unroll
          for (int i = 0; i < 32; i += 4) {
            mx0 = fmax3(mx0, __uint_as_float(r[i]), __uint_as_float(r[i + 1]));
            mx1 = fmax3(mx1, __uint_as_float(r[i + 2]), __uint_as_float(r[i + 3]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (c0 + i < valid) mx0 = fmaxf(mx0, __uint_as_float(r[i]));
        }
      };
      if (ok) {
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          uint32_t ra[32], rb[32];
          tmem_ld32(tS + h2 * 64, ra);
          tmem_ld32(tS + h2 * 64 + 32, rb);
          tmem_ld_wait();
          max_chunk(ra, h2 * 64);
          max_chunk(rb, h2 * 64 + 32);
        }
      }
      const float mx = fmaxf(mx0, mx1);
      if (!ok) break;
      const float m_new = fmaxf(m_used, mx * scale_log2);
      if (!(ok = maybe_rescale(j, m_new))) break;
      // a chunk's P columns were read as scores in an earlier or the same chunk
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        uint32_t ra[32], rb[32];
        tmem_ld32(tS + h2 * 64, ra);
        tmem_ld32(tS + h2 * 64 + 32, rb);
        tmem_ld_wait();
        uint32_t wa[16], wb[16];
        const int pc = 32 * h2;  // packed P columns of this half
        exp_chunk(ra, h2 * 64, valid, wa, l0, l1);
        tmem_st16(tS + pc, wa);
        exp_chunk(rb, h2 * 64 + 32, valid, wb, l0, l1);
        tmem_st16(tS + pc + 16, wb);
      }
      l += l0 + l1;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready(x));
    }
    if (ok && n_kv > 0 && mbar_wait(pv_done(x), (n_kv - 1) & 1, 28)) {
      tc_fence_after();
      const int qrow = it.tile_start + x * BT + row;
      const bool store = qrow < it.seg_len;
      const float inv_l = l > 0.f ? 1.f / l : 0.f;
      __nv_bfloat16* dst = out + ((size_t)(it.seg_start + qrow) * H + h) * D;
      __nv_bfloat16* pdst = (store && o_peer.base) ? peer_row(o_peer, it.seg_start + qrow, h) : nullptr;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(tO + c * 32, r);
        tmem_ld_wait();
        if (store) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = __uint_as_float(r[v * 8 + i]) * inv_l;
            store8(dst + c * 32 + v * 8, o);
            if (pdst) store8(pdst + c * 32 + v * 8, o);
          }
        }
      }
      if (store) lse[(size_t)h * L + it.seg_start + qrow] = (m_used + log2f(l)) * kLn2;
    } else {
      s_abort = 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ============================================================================ fused backward
// One pass, key tiles outer (one CTA = one head x 128 keys of one segment), query tiles inner:
//   S^T  = K Q_i^T,  dP^T = V dO_i^T                        (tcgen05, operands in smem)
//   P^T  = exp2(S^T s log2e - lse_i),  dS^T = P^T (dP^T - Delta_i)   (E warps; lane = key)
//   dV  += P^T dO_i,  dK += dS^T Q_i                        (A = P^T / dS^T straight from TMEM)
//   dQ_i^T = K^T dS^T                                        (tensor core, into the S^T columns)
//   dQ   += dQ_i  via TMA reduce-add of fp32 row blocks      (Q warps; lane = head dim)
// so every score element is exponentiated once and five 128^3 products run per tile pair (the
// two-pass form needs seven and two exponentials).  TMEM: S^T/P^T/dQ^T 0..127, dP^T/dS^T 128..255,
// dV 256..383, dK 384..511.  Warps: 0 TMA, 1 MMA, 2..5 E, 6..9 Q.  dQ accumulates in an fp32
// buffer that a final kernel scales into bf16.
constexpr int FB_THREADS = 320;
constexpr int FB_STAGE = 32 * D * 4;  // 32 query rows of fp32 dQ
constexpr int FB_SMEM = 2 * TILE_BYTES /*K, V*/ + 2 * TILE_BYTES /*Q ring*/ + TILE_BYTES /*dO*/ +
                        TILE_BYTES /*dS^T*/ + 2 * FB_STAGE + 1024 + 256 + 2 * BT * 4;

__global__ void __launch_bounds__(FB_THREADS, 1)
attn_bwd_fused_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap domap,
                      const __grid_constant__ CUtensorMap dqmap, const WorkItem* __restrict__ items, int L, int H,
                      float scale, const float* __restrict__ lse, const float* __restrict__ delta,
                      __nv_bfloat16* __restrict__ dk_out, __nv_bfloat16* __restrict__ dv_out, const PeerRows dk_peer,
                      const PeerRows dv_peer) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + TILE_BYTES;
  uint8_t* sQ = sV + TILE_BYTES;            // 2 slots
  uint8_t* sdO = sQ + 2 * TILE_BYTES;
  uint8_t* sdS = sdO + TILE_BYTES;          // dS^T, [keys][queries] K-major swizzled
  uint8_t* sStage = sdS + TILE_BYTES;       // 2 x [32 q][128 d] fp32
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + 2 * FB_STAGE);
  // kv_full 0, q_full 1-2, q_empty 3-4, do_full 5, do_empty 6, s_full 7, ds_ready 8, ds_free 9,
  // pv_done 10, dq_full 11, dq_drained 12, all_done 13
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);
  volatile int& s_abort = *reinterpret_cast<volatile int*>(bars + 15);
  float (*s_vec)[BT] = reinterpret_cast<float (*)[BT]>(reinterpret_cast<uint8_t*>(bars) + 256);

  const WorkItem it = items[blockIdx.x];
  const int h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_q = (it.seg_len + BT - 1) / BT;
  const float scale_log2 = scale * kLog2e;
  auto B = [&](int i) { return smem_u32(bars + i); };

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < 14; ++i) mbar_init(B(i), (i == 8 || i == 12) ? 4 : 1);  // ds_ready / dq_drained: 4 warps
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t T_S = tmem, T_DP = tmem + 128, T_DV = tmem + 256, T_DK = tmem + 384;
  const int col = h * D;

  if (warp == 0) {
    if (lane == 0) {
      const int r0 = it.seg_start + it.tile_start;
      mbar_expect_tx(B(0), 2 * TILE_BYTES);
      tma_load_2d(smem_u32(sK), &kmap, B(0), col, r0);
      tma_load_2d(smem_u32(sK) + HALF_BYTES, &kmap, B(0), col + 64, r0);
      tma_load_2d(smem_u32(sV), &vmap, B(0), col, r0);
      tma_load_2d(smem_u32(sV) + HALF_BYTES, &vmap, B(0), col + 64, r0);
      for (int i = 0; i < n_q && !s_abort; ++i) {
        const int slot = i & 1;
        const int row = it.seg_start + i * BT;
        if (!mbar_wait(B(3 + slot), ((i >> 1) & 1) ^ 1, 41)) { s_abort = 1; break; }
        mbar_expect_tx(B(1 + slot), TILE_BYTES);
        const uint32_t dq = smem_u32(sQ + slot * TILE_BYTES);
        tma_load_2d(dq, &qmap, B(1 + slot), col, row);
        tma_load_2d(dq + HALF_BYTES, &qmap, B(1 + slot), col + 64, row);
        if (!mbar_wait(B(6), (i & 1) ^ 1, 42)) { s_abort = 1; break; }
        mbar_expect_tx(B(5), TILE_BYTES);
        tma_load_2d(smem_u32(sdO), &domap, B(5), col, row);
        tma_load_2d(smem_u32(sdO) + HALF_BYTES, &domap, B(5), col + 64, row);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t id_kk = idesc_bf16_f32(128, 128, 0, 0);  // S^T, dP^T: both K-major over D
      const uint32_t id_tm = idesc_bf16_f32(128, 128, 0, 1);  // dV, dK: A from TMEM, B MN-major
      const uint32_t id_mm = idesc_bf16_f32(128, 128, 1, 1);  // dQ^T: A = K^T, B = dS^T, both MN-major
      const uint32_t k = smem_u32(sK), v = smem_u32(sV), dO = smem_u32(sdO), dS = smem_u32(sdS);
      bool ok = mbar_wait(B(0), 0, 43);
      for (int i = 0; i < n_q && ok; ++i) {
        const int slot = i & 1;
        const uint32_t q = smem_u32(sQ + slot * TILE_BYTES);
        if (!(ok = mbar_wait(B(1 + slot), (i >> 1) & 1, 44))) break;
        if (!(ok = mbar_wait(B(5), i & 1, 45))) break;
        if (i > 0 && !(ok = mbar_wait(B(12), (i - 1) & 1, 46))) break;  // dQ^T(i-1) drained
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma_bf16_ss(T_S, desc_kmajor(k, kk), desc_kmajor(q, kk), id_kk, kk > 0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) mma_bf16_ss(T_DP, desc_kmajor(v, kk), desc_kmajor(dO, kk), id_kk, kk > 0);
        mma_commit(B(7));
        if (!(ok = mbar_wait(B(8), i & 1, 47))) break;  // P^T, dS^T in TMEM and dS^T in smem
        tc_fence_after();
        // dV += P^T dO_i ; dK += dS^T Q_i  (K = 128 queries, 8 columns of packed bf16 per step)
#pragma unroll
        for (int kk = 0; kk < BT / 16; ++kk)
          mma_bf16_ts(T_DV, T_S + kk * 8, desc_mnmajor(dO, kk), id_tm, (i > 0) || (kk > 0));
        mma_commit(B(6));  // dO slot free
#pragma unroll
        for (int kk = 0; kk < BT / 16; ++kk)
          mma_bf16_ts(T_DK, T_DP + kk * 8, desc_mnmajor(q, kk), id_tm, (i > 0) || (kk > 0));
        mma_commit(B(3 + slot));  // Q slot free
        mma_commit(B(10));
        if (!(ok = mbar_wait(B(10), i & 1, 48))) break;  // P^T read before dQ^T overwrites its columns
        tc_fence_after();
        // dQ_i^T = K^T dS^T  (M = D, N = queries, K = keys)
#pragma unroll
        for (int kk = 0; kk < BT / 16; ++kk) mma_bf16_ss(T_S, desc_mnmajor(k, kk), desc_mnmajor(dS, kk), id_mm, kk > 0);
        mma_commit(B(11));
        mma_commit(B(9));  // dS^T smem free
      }
      mma_commit(B(13));
      if (!ok) s_abort = 1;
    }
  } else if (warp < 6) {
    // ------------------------------------------------ E warps: P^T and dS^T (lane = key row)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const bool row_valid = it.tile_start + row < it.seg_len;
    const int tid = threadIdx.x - 64;
    bool ok = true;
    // LSE / Delta of query tile i are loaded from global memory one tile ahead (registers), so their
    // latency overlaps the previous tile's work instead of stalling every tile
    auto fetch = [&](int i, float& lv, float& dv) {
      const int qi = i * BT + tid;
      const bool in = i < n_q && qi < it.seg_len;
      lv = in ? lse[(size_t)h * L + it.seg_start + qi] * kLog2e : 0.f;
      dv = in ? delta[(size_t)h * L + it.seg_start + qi] : 0.f;
    };
    float next_l, next_d;
    fetch(0, next_l, next_d);
    for (int i = 0; i < n_q; ++i) {
      const int valid_q = min(BT, it.seg_len - i * BT);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      s_vec[0][tid] = next_l;
      s_vec[1][tid] = next_d;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      fetch(i + 1, next_l, next_d);
      // no break between the named barriers: after a bounded wait gave up the warp keeps meeting
      // them (skipping its work), so its group partners never wait on it forever
      if (ok) ok = mbar_wait(B(7), i & 1, 49);
      if (ok && i > 0) ok = mbar_wait(B(9), (i - 1) & 1, 50);  // dQ^T(i-1) has read dS^T smem
      if (!ok) continue;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32], y[32];
        tmem_ld32(T_S + lane_off + c * 32, r);
        tmem_ld32(T_DP + lane_off + c * 32, y);
        tmem_ld_wait();
        uint32_t wp[16], wd[16];
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
          float pv[2], dsv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int cc = c * 32 + j + e;
            const bool on = cc < valid_q && row_valid;
            const float p = on ? fast_exp2(__uint_as_float(r[j + e]) * scale_log2 - s_vec[0][cc]) : 0.f;
            pv[e] = p;
            dsv[e] = p * (__uint_as_float(y[j + e]) - s_vec[1][cc]);
          }
          wp[j >> 1] = pack_bf16(pv[0], pv[1]);
          wd[j >> 1] = pack_bf16(dsv[0], dsv[1]);
        }
        // columns [16c, 16c + 16) were read in chunk c or earlier
        tmem_st16(T_S + lane_off + c * 16, wp);
        tmem_st16(T_DP + lane_off + c * 16, wd);
        store_row32_swizzled(sdS, row, c * 32, wd);
      }
      tmem_st_wait();
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(B(8));
    }
    // dV, dK rows of this key tile
    if (ok && n_q > 0 && mbar_wait(B(13), 0, 51)) {
      tc_fence_after();
      const int g = it.seg_start + it.tile_start + row;
      const size_t grow = (size_t)g * H + h;
      for (int which = 0; which < 2; ++which) {
        const uint32_t tacc = (which == 0 ? T_DK : T_DV) + lane_off;
        const float mul = which == 0 ? scale : 1.f;
        const PeerRows& pr = which == 0 ? dk_peer : dv_peer;
        __nv_bfloat16* dst = pr.base ? (row_valid ? peer_row(pr, g, h) : nullptr)
                                     : (which == 0 ? dk_out : dv_out) + grow * D;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          tmem_ld32(tacc + c * 32, r);
          tmem_ld_wait();
          if (row_valid) {
#pragma unroll
            for (int vv = 0; vv < 4; ++vv) {
              float o[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) o[e] = __uint_as_float(r[vv * 8 + e]) * mul;
              store8(dst + c * 32 + vv * 8, o);
            }
          }
        }
      }
    } else {
      s_abort = 1;
    }
  } else {
    // ------------------------------------------------ Q warps: dQ^T -> fp32 reduce-add (lane = d)
    const int quarter = warp & 3;
    const int d = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int qt = threadIdx.x - 192;  // 0..127
    int n_used = 0;
    bool ok = true;
    // the four drain warps meet their named barrier the same number of times whatever happens: a
    // bounded wait that gave up only turns the data movement off
    for (int i = 0; i < n_q; ++i) {
      if (ok && !(ok = mbar_wait(B(11), i & 1, 52))) s_abort = 1;
      if (ok) tc_fence_after();
      uint32_t r[4][32];
      if (ok) {
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(T_S + lane_off + c * 32, r[c]);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(B(12));  // the S^T columns may be rewritten
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float* st = reinterpret_cast<float*>(sStage + (n_used & 1) * FB_STAGE);
        if (n_used >= 2 && qt == 0) bulk_wait_read<1>();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (ok) {
#pragma unroll
          for (int qq = 0; qq < 32; ++qq) st[qq * D + d] = __uint_as_float(r[c][qq]);
        }
        fence_async_shared();
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (qt == 0 && ok) tma_reduce_add_2d(&dqmap, smem_u32(st), col, it.seg_start + i * BT + c * 32);
        if (qt == 0) bulk_commit();
        ++n_used;
      }
    }
    if (qt == 0) bulk_wait_all();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dq = scale * dq_acc (fp32 -> bf16), 8 elements per thread
// With `dq_peer` on, element (row g, head h, d) goes to its token owner instead (the reverse
// all-to-all of dQ) and rows at or beyond n_valid are skipped (the owners zero their padding).
__global__ void attn_dq_convert_kernel(const float* __restrict__ acc, size_t n8, float scale,
                                       __nv_bfloat16* __restrict__ dq, const PeerRows dq_peer, int H, int n_valid) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const float4 a = reinterpret_cast<const float4*>(acc)[2 * i];
  const float4 b = reinterpret_cast<const float4*>(acc)[2 * i + 1];
  float v[8] = {a.x * scale, a.y * scale, a.z * scale, a.w * scale, b.x * scale, b.y * scale, b.z * scale, b.w * scale};
  if (dq_peer.base == nullptr) {
    store8(dq + 8 * i, v);
    return;
  }
  const size_t e = 8 * i;
  const int g = (int)(e / ((size_t)H * D));
  if (g >= n_valid) return;
  const int rem = (int)(e - (size_t)g * H * D);
  store8(peer_row(dq_peer, g, rem / D) + (rem % D), v);
}

// Ulysses backward prologue: dO of global row g and head h (heads [head_base, head_base + H) of
// this rank) is read from its token owner (the all-to-all of dO, peer loads) into the local
// head-sharded dO, and Delta[h, g] = sum_d dO * O is formed on the way.  One warp per (row, head);
// rows at or beyond n_valid are zeroed.
__global__ void attn_bwd_gather_delta_kernel(const __nv_bfloat16* __restrict__ o, const PeerRows do_src, int L,
                                             int H, int n_valid, __nv_bfloat16* __restrict__ dout,
                                             float* __restrict__ delta) {
  const int lane = threadIdx.x & 31;
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= L * H) return;
  const int row = w / H, h = w % H;
  const size_t base = ((size_t)row * H + h) * D + lane * 4;
  uint2 b = make_uint2(0u, 0u);
  if (row < n_valid) b = *reinterpret_cast<const uint2*>(peer_row(do_src, row, h) + lane * 4);
  *reinterpret_cast<uint2*>(dout + base) = b;
  const uint2 a = *reinterpret_cast<const uint2*>(o + base);
  const float2 a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.x));
  const float2 a1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.y));
  const float2 b0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.x));
  const float2 b1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.y));
  float s = a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y;
  s = warp_sum(s);
  if (lane == 0) delta[(size_t)h * L + row] = s;
}

// Delta[h, i] = sum_d dO[i, h, d] * O[i, h, d]  (fp32), one warp per (row, head).
__global__ void attn_bwd_delta_kernel(const __nv_bfloat16* __restrict__ o, const __nv_bfloat16* __restrict__ dout,
                                      int L, int H, float* __restrict__ delta) {
  const int lane = threadIdx.x & 31;
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (w >= L * H) return;
  const int row = w / H, h = w % H;
  const size_t base = ((size_t)row * H + h) * D + lane * 4;
  const uint2 a = *reinterpret_cast<const uint2*>(o + base);
  const uint2 b = *reinterpret_cast<const uint2*>(dout + base);
  const float2 a0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.x));
  const float2 a1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.y));
  const float2 b0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.x));
  const float2 b1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&b.y));
  float s = a0.x * b0.x + a0.y * b0.y + a1.x * b1.x + a1.y * b1.y;
  s = warp_sum(s);
  if (lane == 0) delta[(size_t)h * L + row] = s;
}

// ---------------------------------------------------------------------------- host helpers
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

const char* make_qkv_map(CUtensorMap* m, const void* base, int L, int H, int box_rows = BT) {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess || !ptr)
      return "cuTensorMapEncodeTiled is unavailable";
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  if (reinterpret_cast<uintptr_t>(base) % 16) return "attention: tensor base must be 16-byte aligned";
  cuuint64_t dims[2] = {(cuuint64_t)H * D, (cuuint64_t)L};
  cuuint64_t strides[1] = {(cuuint64_t)H * D * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? nullptr : "cuTensorMapEncodeTiled failed (attention)";
}

// fp32 [L, H*D] accumulator map for the dQ reduce-add: boxes of 32 rows x 128 columns, no swizzle.
const char* make_dq_map(CUtensorMap* m, const float* base, int L, int H) {
  static EncodeTiledFn fn = nullptr;
  if (fn == nullptr) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess || !ptr)
      return "cuTensorMapEncodeTiled is unavailable";
    fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  if (reinterpret_cast<uintptr_t>(base) % 16) return "attention: dq accumulator must be 16-byte aligned";
  cuuint64_t dims[2] = {(cuuint64_t)H * D, (cuuint64_t)L};
  cuuint64_t strides[1] = {(cuuint64_t)H * D * 4};
  cuuint32_t box[2] = {(cuuint32_t)D, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? nullptr : "cuTensorMapEncodeTiled failed (dq accumulator)";
}

// Key-tile-outer fused backward into dq_acc / dk / dv.
const char* run_bwd_single_pass(const void* q, const void* k, const void* v, const void* dout, const float* lse,
                                const float* delta, const int* items_kv, int n_items_kv, int L, int H, float scale,
                                float* dq_acc, __nv_bfloat16* dk, __nv_bfloat16* dv, const PeerRows& dk_peer,
                                const PeerRows& dv_peer, cudaStream_t s) {
  CUtensorMap qm, km, vm, dom, dqm;
  const char* e;
  if ((e = make_qkv_map(&qm, q, L, H)) || (e = make_qkv_map(&km, k, L, H)) || (e = make_qkv_map(&vm, v, L, H)) ||
      (e = make_qkv_map(&dom, dout, L, H)) || (e = make_dq_map(&dqm, dq_acc, L, H)))
    return e;
  static bool attr = false;
  if (!attr) {
    if (cudaFuncSetAttribute(attn_bwd_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FB_SMEM) !=
        cudaSuccess)
      return "attention: cannot set smem size (fused backward)";
    attr = true;
  }
  if (cudaMemsetAsync(dq_acc, 0, (size_t)L * H * D * sizeof(float), s) != cudaSuccess) return "dq memset failed";
  if (n_items_kv > 0)
    attn_bwd_fused_kernel<<<dim3(n_items_kv, H), FB_THREADS, FB_SMEM, s>>>(
        qm, km, vm, dom, dqm, reinterpret_cast<const WorkItem*>(items_kv), L, H, scale, lse, delta, dk, dv, dk_peer,
        dv_peer);
  return cudaGetLastError() == cudaSuccess ? nullptr : "attention backward launch failed";
}

// Forward kernel: 1 = in-order MMA issue (default), 0 = PV completion awaited before the next score GEMM.
int g_fwd_inorder = 1;

}  // namespace attn

void attn_set_forward_variant(int v) { attn::g_fwd_inorder = v ? 1 : 0; }
int attn_get_variant(int backward) { return backward ? 0 : attn::g_fwd_inorder; }

const char* launch_attn_fwd(const void* q, const void* k, const void* v, const int* items, int n_items, int L, int H,
                            int head_dim, float scale, void* out, float* lse, cudaStream_t s, const uint64_t* o_peer,
                            int cp, int head_base, int H_total) {
  using namespace attn;
  const PeerRows opr{o_peer, cp, head_base, H_total};
  if (o_peer && (cp < 1 || head_base < 0 || head_base + H > H_total)) return "attention: bad peer head range";
  if (head_dim != D) return "attention: head_dim must be 128";
  if (n_items == 0) return nullptr;
  CUtensorMap qm, km, vm;
  const char* e;
  if ((e = make_qkv_map(&qm, q, L, H)) || (e = make_qkv_map(&km, k, L, H)) || (e = make_qkv_map(&vm, v, L, H))) return e;
  typedef void (*FwdKernel)(CUtensorMap, CUtensorMap, CUtensorMap, const WorkItem*, int, int, float, __nv_bfloat16*,
                            float*, PeerRows);
  static const FwdKernel variants[2] = {attn_fwd_kernel<false>, attn_fwd_kernel<true>};
  static bool attr[2] = {};
  const int var = g_fwd_inorder;
  if (!attr[var]) {
    if (cudaFuncSetAttribute(variants[var], cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM) != cudaSuccess)
      return "attention: cannot set smem size";
    attr[var] = true;
  }
  dim3 grid(n_items, H);
  auto kern = variants[var];
  kern<<<grid, FWD_THREADS, FWD_SMEM, s>>>(qm, km, vm, reinterpret_cast<const WorkItem*>(items), L, H, scale * kLog2e,
                                           (__nv_bfloat16*)out, lse, opr);
  return cudaGetLastError() == cudaSuccess ? nullptr : "attention forward launch failed";
}

const char* launch_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                            const float* lse, const int* items_q, int n_items_q, const int* items_kv, int n_items_kv,
                            int L, int H, int head_dim, float scale, float* delta, void* dq, void* dk, void* dv,
                            float* dq_acc, cudaStream_t s) {
  using namespace attn;
  if (head_dim != D) return "attention: head_dim must be 128";
  const int warps = L * H;
  attn_bwd_delta_kernel<<<(warps * 32 + 255) / 256, 256, 0, s>>>((const __nv_bfloat16*)o,
                                                                 (const __nv_bfloat16*)dout, L, H, delta);
  if (dq_acc == nullptr) return "attention backward: an fp32 dQ accumulator is required";
  const char* e;
  if ((e = run_bwd_single_pass(q, k, v, dout, lse, delta, items_kv, n_items_kv, L, H, scale, dq_acc,
                               (__nv_bfloat16*)dk, (__nv_bfloat16*)dv, PeerRows{nullptr, 1, 0, H},
                               PeerRows{nullptr, 1, 0, H}, s)))
    return e;
  const size_t n8 = (size_t)L * H * D / 8;
  attn_dq_convert_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(dq_acc, n8, scale, (__nv_bfloat16*)dq,
                                                                       PeerRows{nullptr, 1, 0, H}, H, L);
  return cudaGetLastError() == cudaSuccess ? nullptr : "attention backward launch failed";
}

int attn_error_flag(bool reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, sm100::g_error_flag, sizeof(int));
  if (reset) {
    int z = 0;
    cudaMemcpyToSymbol(sm100::g_error_flag, &z, sizeof(int));
  }
  return v;
}

// Ulysses context-parallel backward over the full sequence for this rank's H heads: dO is pulled
// from its token owners while Delta is formed, the fused kernel writes dK / dV rows straight to
// their token owners, and the dQ conversion does the same for dQ.  q/k/v/o/lse/dout_head are this
// rank's head-sharded buffers (local memory); the *_peer tables hold every cp-rank's address of its
// token-sharded [rows, H_total, D] buffer.
const char* launch_attn_bwd_cp(const void* q, const void* k, const void* v, const void* o, const float* lse,
                               const int* items_kv, int n_items_kv, int L, int H, int head_dim, float scale,
                               int n_valid, float* delta, void* dout_head, float* dq_acc, const uint64_t* do_peer,
                               const uint64_t* dq_peer, const uint64_t* dk_peer, const uint64_t* dv_peer, int cp,
                               int head_base, int H_total, cudaStream_t s) {
  using namespace attn;
  if (head_dim != D) return "attention: head_dim must be 128";
  if (cp < 1 || head_base < 0 || head_base + H > H_total) return "attention: bad peer head range";
  const PeerRows dsrc{do_peer, cp, head_base, H_total};
  const int warps = L * H;
  attn_bwd_gather_delta_kernel<<<(warps * 32 + 255) / 256, 256, 0, s>>>((const __nv_bfloat16*)o, dsrc, L, H, n_valid,
                                                                        (__nv_bfloat16*)dout_head, delta);
  const char* e = run_bwd_single_pass(q, k, v, dout_head, lse, delta, items_kv, n_items_kv, L, H, scale, dq_acc,
                                      nullptr, nullptr, PeerRows{dk_peer, cp, head_base, H_total},
                                      PeerRows{dv_peer, cp, head_base, H_total}, s);
  if (e) return e;
  const size_t n8 = (size_t)L * H * D / 8;
  attn_dq_convert_kernel<<<(unsigned)((n8 + 255) / 256), 256, 0, s>>>(dq_acc, n8, scale, nullptr,
                                                                       PeerRows{dq_peer, cp, head_base, H_total}, H,
                                                                       n_valid);
  return cudaGetLastError() == cudaSuccess ? nullptr : "attention context-parallel backward launch failed";
}

}  // namespace pan

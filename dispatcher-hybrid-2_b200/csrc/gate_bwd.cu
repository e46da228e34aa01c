// Backward of the gate readout (the reference op dispatcher::gate_preacts_bwd,
// fused_gates.py:96-173 and 225-263).  Given dP_x = dL/d pre_x (x = i, f, r),
// each (b, T, n_lv, H):
//   x(t,k)    = A(t,k) + m_l(t) B(t - 2^l, k)        (bf16, as the forward)
//   h(t,k)    = relu(x)^2                           (bf16)
//   dh(t,k)   = sum_j dP(t,l,j) W_l(j,k)            j = (x, h), 3H of them
//   dx(t,k)   = 2 relu(x) dh                        (fp32)
//   dA(t,k)  += dx;   dB(t - 2^l, k) += m_l(t) dx
//   dW_l(j,k)+= sum_t dP(t,l,j) h(t,k);   db_l(j) += sum_t dP(t,l,j)
//
// One CTA per (sequence, 128 positions); 64-column slices of the gate-hidden
// width outermost, levels innermost, two pipeline stages.  Warp roles:
//   warp 0      TMA: the A tile of a slice, the B tile shifted by 2^l and the
//               W_l^T slice (W pre-transposed and padded to 64 gate rows) of
//               each (slice, level), and at 16 heads the step's dP rows
//               (3 x 128 positions x 32 bytes)
//   warp 1      tcgen05.mma, no mbarrier waits (a named-barrier handoff from
//               warp 10): dh = dP . W_l^T (M=128 positions, N=64, K=48) and
//               dW^T = dP^T . h^T (M=128 gate rows, 48 used, N=64, K=128
//               positions), both into TMEM; dW^T reads the dP tile and the h
//               tile MN-major, i.e. with positions as K, so no transposed
//               copy is ever written
//   warps 2-9   two threads per position (32 columns each): write the
//               position's dP row and h row into shared memory (16-byte
//               stores), recompute x and relu(x);
//               then, one stage later, read dh back and accumulate dA in
//               registers over the levels (stored once per slice: only this
//               CTA writes these positions), add dB, dW and db atomically
//   warp 10     mbarrier waits for warp 1
// dh's operands are K-major, dW^T's MN-major, all with the 128-byte swizzle
// (rows of 128 bytes, 16-byte chunk c of row r at c ^ (r & 7)).  Every wait is
// bounded; after a failed wait a thread skips later waits but keeps every
// handoff, so nothing blocks.
#include "common.cuh"
#include "tma.cuh"

namespace dh {
namespace {

constexpr int kGbT = 128;                      // positions per CTA
constexpr int kGbK = 64;                       // gate-hidden columns per slice
constexpr int kGbJ = 64;                       // gate rows (3H) padded
constexpr int kGbThreads = 352;
constexpr int kGbWaiterWarp = 10;
constexpr int kGbHandoffBar = 1;
constexpr int kGbTile = kGbT * 128;            // 16 KB: 128 rows of 128 bytes
// per stage: dP (t x j) 16 KB, a zero tile 16 KB (gate rows 64..127 of the
// dW^T MMA's M = 128), h (t x k) 16 KB
constexpr int kGbStageBytes = 3 * kGbTile;
constexpr int kGbDpIn = 3 * kGbT * 32;         // 12 KB: dP rows of one step (16 heads)
constexpr int kGbSmem = 1024 + 2 * kGbStageBytes + 2 * kGbTile /*A*/ + 2 * kGbTile /*B*/ +
                        2 * (kGbK * 128) /*W^T*/ + 2 * kGbDpIn + 256;
constexpr int kGbTmemCols = 256;               // per stage: dh 64 + dW^T 64 (x2 stages)

struct GbArgs {
  int B, T, H, n_lv, gh, mask_L;
  const uint8_t* mask;                         // (B, T, mask_L) or null
  const __nv_bfloat16 *dpi, *dpf, *dpr;        // (B, T, n_lv, H)
  float *dA, *dB;                              // (B, T, gh)
  float *dWi, *dWf, *dWr;                      // (n_lv, H, gh)
  float *dbi, *dbf, *dbr;                      // (n_lv, H)
  int* err;
};

__device__ __forceinline__ void gb_red4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

__device__ __forceinline__ uint32_t b2u(__nv_bfloat162 v) {
  uint32_t u;
  memcpy(&u, &v, 4);
  return u;
}

// byte offset of element (row, col) in a 128-byte-row tile with the 128B swizzle
__device__ __forceinline__ uint32_t sw_off(int row, int col) {
  return (uint32_t)(row * 128 + ((((col >> 3) ^ (row & 7)) & 7) << 4) + (col & 7) * 2);
}

__device__ __forceinline__ bool gb_handoff(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 64, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "n"(kGbHandoffBar)
      : "memory");
  return r != 0;
}

// MN-major 128B-swizzled operand: each 128-byte row is one K index (here a
// position) holding 64 MN elements; 8-row groups are 1024 B apart (SBO) and
// the next 64 MN elements start lbo bytes on (LBO)
__device__ __forceinline__ uint64_t mn_sw128_desc(uint32_t smem_addr, uint32_t lbo) {
  return (sw128_desc(smem_addr) & ~(uint64_t(0x3FFF) << 16)) | ((uint64_t)(lbo >> 4) << 16);
}

// shared memory: two stages of [dP | zero tile | h], then the
// A tiles, the B tiles, the W^T tiles and the dP row copies (two of each),
// then the barriers
struct GbSmem {
  uint8_t* base;
  __device__ __forceinline__ uint8_t* stage(int s) const { return base + s * kGbStageBytes; }
  __device__ __forceinline__ uint8_t* a(int s) const { return base + 2 * kGbStageBytes + s * kGbTile; }
  __device__ __forceinline__ uint8_t* b(int s) const {
    return base + 2 * kGbStageBytes + 2 * kGbTile + s * kGbTile;
  }
  __device__ __forceinline__ uint8_t* wt(int s) const {
    return base + 2 * kGbStageBytes + 4 * kGbTile + s * (kGbK * 128);
  }
  __device__ __forceinline__ uint8_t* dpin(int s) const {
    return base + 2 * kGbStageBytes + 4 * kGbTile + 2 * (kGbK * 128) + s * kGbDpIn;
  }
  __device__ __forceinline__ uint8_t* end() const {
    return base + 2 * kGbStageBytes + 4 * kGbTile + 2 * (kGbK * 128) + 2 * kGbDpIn;
  }
};

__device__ __forceinline__ uint8_t* st_dp(uint8_t* s) { return s; }
__device__ __forceinline__ uint8_t* st_zero(uint8_t* s) { return s + kGbTile; }
__device__ __forceinline__ uint8_t* st_h(uint8_t* s) { return s + 2 * kGbTile; }

__global__ void __launch_bounds__(kGbThreads, 1)
    gate_bwd_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                    const __grid_constant__ CUtensorMap tmW,
                    const __grid_constant__ CUtensorMap tmDi,
                    const __grid_constant__ CUtensorMap tmDf,
                    const __grid_constant__ CUtensorMap tmDr, GbArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const GbSmem S{smem};
  uint64_t* bars = reinterpret_cast<uint64_t*>(S.end());
  uint64_t* a_full = bars;          // [2] A tile of slice kc, by kc & 1
  uint64_t* a_empty = bars + 2;     // [2]
  uint64_t* tb_full = bars + 4;     // [2] B tile + W^T (+ dP rows) of iteration i, by i & 1
  uint64_t* ops_full = bars + 6;    // [2] dP and h written
  uint64_t* mma_done = bars + 8;    // [2] both contractions of iteration i complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kGbT, b = blockIdx.y;
  const int nk = g.gh / kGbK, nl = g.n_lv, H = g.H, H3 = 3 * g.H;
  const int iters = nk * nl;
  const bool dp_tma = H == 16;      // dP rows arrive by TMA (32-byte rows)

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 8);
      mbar_init(&tb_full[s], 1);
      mbar_init(&ops_full[s], 8);
      mbar_init(&mma_done[s], 1);
    }
    fence_barrier_init();
  }
  // dP columns >= 3H and the zero tile stay zero: the dW^T MMA reads all 128
  // gate rows of its M (rows 64..127 from the zero tile)
  for (int s = 0; s < 2; ++s) {
    uint4* z = reinterpret_cast<uint4*>(st_zero(S.stage(s)));
    for (int i = threadIdx.x; i < kGbTile / 16; i += blockDim.x) z[i] = make_uint4(0, 0, 0, 0);
    uint4* zp = reinterpret_cast<uint4*>(st_dp(S.stage(s)));
    for (int i = threadIdx.x; i < kGbTile / 16; i += blockDim.x) zp[i] = make_uint4(0, 0, 0, 0);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) {
    tmem_alloc(tmem_slot, kGbTmemCols);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmW);
    if (dp_tma) {
      prefetch_tmap(&tmDi);
      prefetch_tmap(&tmDf);
      prefetch_tmap(&tmDr);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      bool ok = true;
      for (int i = 0; i < iters && ok; ++i) {
        const int kc = i / nl, l = i - kc * nl, s = i & 1;
        if (l == 0) {
          if (kc >= 2) ok = ok && mbar_wait(&a_empty[kc & 1], (uint32_t)(((kc >> 1) - 1) & 1), g.err);
          if (!ok) break;
          mbar_arrive_expect_tx(&a_full[kc & 1], kGbTile);
          tma_load_3d(&tmA, &a_full[kc & 1], S.a(kc & 1), kc * kGbK, t0, b);
        }
        // stage s was last used by iteration i - 2: its MMAs must be done
        if (i >= 2) ok = ok && mbar_wait(&mma_done[s], (uint32_t)(((i >> 1) - 1) & 1), g.err);
        if (!ok) break;
        mbar_arrive_expect_tx(&tb_full[s], kGbTile + kGbK * 128 + (dp_tma ? kGbDpIn : 0));
        tma_load_3d(&tmB, &tb_full[s], S.b(s), kc * kGbK, t0 - (1 << l), b);
        tma_load_2d(&tmW, &tb_full[s], S.wt(s), 0, l * g.gh + kc * kGbK);
        if (dp_tma) {  // box (16 heads, 1 level, 128 positions, 1 sequence), rows past T read 0
          tma_load_4d(&tmDi, &tb_full[s], S.dpin(s), 0, l, t0, b);
          tma_load_4d(&tmDf, &tb_full[s], S.dpin(s) + kGbT * 32, 0, l, t0, b);
          tma_load_4d(&tmDr, &tb_full[s], S.dpin(s) + 2 * kGbT * 32, 0, l, t0, b);
        }
      }
      // drain: every issued copy has landed before exit
      if (iters > 0) mbar_wait(&tb_full[(iters - 1) & 1], (uint32_t)(((iters - 1) >> 1) & 1), nullptr, 1u << 20);
      if (iters > 1) mbar_wait(&tb_full[iters & 1], (uint32_t)(((iters - 2) >> 1) & 1), nullptr, 1u << 20);
      if (nk > 0) mbar_wait(&a_full[(nk - 1) & 1], (uint32_t)(((nk - 1) >> 1) & 1), nullptr, 1u << 20);
    }
  } else if (warp == 1) {  // ---------------- MMA issue
    const uint32_t id_dh = idesc_bf16(kGbT, kGbK);
    const uint32_t id_dw = idesc_bf16(128, kGbK) | (1u << 15) | (1u << 16);  // A, B MN-major
    bool ok = true;
    for (int i = 0; i < iters; ++i) {
      const int s = i & 1;
      ok = gb_handoff(ok);  // the waiter saw this stage's operands written
      tc_fence_after();
      if (ok && lane == 0) {
        uint8_t* st = S.stage(s);
        const uint32_t dp = smem_u32(st_dp(st)), hp = smem_u32(st_h(st)), wt = smem_u32(S.wt(s));
        const uint32_t d_dh = tmem + (uint32_t)(s * 128), d_dw = d_dh + 64;
#pragma unroll
        for (int kk = 0; kk < 3; ++kk)  // K = 48 gate rows (3H <= 48; rows past 3H are 0)
          umma_bf16(d_dh, sw128_desc(dp + kk * 32), sw128_desc(wt + kk * 32), id_dh, kk != 0);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // K = 128 positions, 16 rows (2 KB) per instruction
          umma_bf16(d_dw, mn_sw128_desc(dp + kk * 2048, kGbTile), mn_sw128_desc(hp + kk * 2048, kGbTile),
                    id_dw, kk != 0);
        umma_commit(&mma_done[s]);
      }
      __syncwarp();
    }
  } else if (warp == kGbWaiterWarp) {  // ---------------- waiter
    bool ok = true;
    for (int i = 0; i < iters; ++i) {
      ok = ok && mbar_wait(&ops_full[i & 1], (uint32_t)((i >> 1) & 1), g.err);
      ok = gb_handoff(ok);
    }
  } else {  // ---------------- builders / epilogue, warps 2..9
    const int q = warp & 3;                 // TMEM lane quadrant
    const int half = (warp - 2) >> 2;       // which 32 columns of the slice
    const int r = q * 32 + lane;            // tile row = position t0 + r = TMEM lane
    const int t = t0 + r;
    const bool row_ok = t < g.T;
    bool ok = true;
    float dacc[32];
#pragma unroll
    for (int e = 0; e < 32; ++e) dacc[e] = 0.f;
    uint32_t rx0[16], rx1[16];              // relu(x) of the two stages in flight, bf16x2

    // one (slice, level) step: operands of iteration i into stage S, then the
    // epilogue of iteration i - 1 (stage 1 - S)
    auto build = [&](int i, uint32_t (&rx)[16]) {
      const int kc = i / nl, l = i - kc * nl, s = i & 1;
      const int sh = 1 << l;
      uint8_t* st = S.stage(s);
      if (i >= 2) ok = ok && mbar_wait(&mma_done[s], (uint32_t)(((i >> 1) - 1) & 1), g.err);
      if (l == 0) ok = ok && mbar_wait(&a_full[kc & 1], (uint32_t)((kc >> 1) & 1), g.err);
      ok = ok && mbar_wait(&tb_full[s], (uint32_t)((i >> 1) & 1), g.err);
      // source mask of this row at level l (wrap handled by the TMA zeros)
      bool m = row_ok && t >= sh;
      if (g.mask && m) m = g.mask[((size_t)b * g.T + t) * g.mask_L + l] != 0;
      // dP row: this thread's 24 of the 3H <= 48 gate rows (half 0: j 0..23)
      {
        uint32_t v[12];
#pragma unroll
        for (int e = 0; e < 12; ++e) v[e] = 0u;
        if (row_ok && dp_tma) {
          // the three 32-byte dP rows of this position, copied in by TMA: half
          // 0 takes dPi and the first half of dPf, half 1 the rest
          const uint8_t* rows = S.dpin(s) + r * 32;
          const uint4* pi = reinterpret_cast<const uint4*>(rows);
          const uint4* pf = reinterpret_cast<const uint4*>(rows + kGbT * 32);
          const uint4* pr = reinterpret_cast<const uint4*>(rows + 2 * kGbT * 32);
          const uint4 u0 = half ? pf[1] : pi[0], u1 = half ? pr[0] : pi[1], u2 = half ? pr[1] : pf[0];
          v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
          v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
          v[8] = u2.x; v[9] = u2.y; v[10] = u2.z; v[11] = u2.w;
        } else if (row_ok) {
          const size_t o = (((size_t)b * g.T + t) * nl + l) * H;
#pragma unroll
          for (int e = 0; e < 24; e += 2) {
            const int j = half * 24 + e;
            float f2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int jj = j + u;
              float val = 0.f;
              if (jj < H3) {
                const int x = jj / H, hh = jj - x * H;
                const __nv_bfloat16* src = x == 0 ? g.dpi : (x == 1 ? g.dpf : g.dpr);
                val = bf2f(src[o + hh]);
              }
              f2[u] = val;
            }
            v[e / 2] = pack2(f2[0], f2[1]);
          }
        }
        // row r of dP (t x j): 3 chunks of 8 columns
        uint8_t* dpb = st_dp(st);
#pragma unroll
        for (int c = 0; c < 3; ++c)
          *reinterpret_cast<uint4*>(dpb + sw_off(r, half * 24 + c * 8)) =
              make_uint4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
        // db_l: column sums over the tile's rows, once per level (slice 0)
        if (kc == 0) {
#pragma unroll
          for (int e = 0; e < 24; ++e) {
            float x = __uint_as_float((v[e >> 1] >> ((e & 1) * 16)) << 16);
            x = warp_sum(x);
            const int jj = half * 24 + e;
            if (lane == 0 && jj < H3 && x != 0.f) {
              const int xx = jj / H, hh = jj - xx * H;
              float* db = xx == 0 ? g.dbi : (xx == 1 ? g.dbf : g.dbr);
              asm volatile("red.global.add.f32 [%0], %1;" ::"l"(db + l * H + hh), "f"(x) : "memory");
            }
          }
        }
      }
      // x = A + m B(t - 2^l) in bf16, relu, h = relu^2 -> row r of h
      {
        const uint8_t* arow = S.a(kc & 1) + r * 128;
        const uint8_t* brow = S.b(s) + r * 128;
        const __nv_bfloat162 m2 = __floats2bfloat162_rn(m ? 1.f : 0.f, m ? 1.f : 0.f);
        const __nv_bfloat162 z2 = __floats2bfloat162_rn(0.f, 0.f);
        uint8_t* hrow = st_h(st);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int chunk = half * 4 + c;
          uint4 av = *reinterpret_cast<const uint4*>(arow + ((chunk ^ (r & 7)) << 4));
          uint4 bv = *reinterpret_cast<const uint4*>(brow + ((chunk ^ (r & 7)) << 4));
          const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&av);
          const __nv_bfloat162* b2 = reinterpret_cast<const __nv_bfloat162*>(&bv);
          uint32_t hb[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 x = __hfma2(m2, b2[e], a2[e]);
            x = __hmax2(x, z2);
            rx[c * 4 + e] = b2u(x);
            hb[e] = b2u(__hmul2_rn(x, x));
          }
          *reinterpret_cast<uint4*>(hrow + sw_off(r, chunk * 8)) = make_uint4(hb[0], hb[1], hb[2], hb[3]);
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ops_full[s]);
        if (l == nl - 1) mbar_arrive(&a_empty[kc & 1]);  // the slice's A tile is no longer read
      }
    };

    auto epilogue = [&](int i, const uint32_t (&rx)[16]) {
      const int kc = i / nl, l = i - kc * nl, s = i & 1;
      const int sh = 1 << l;
      ok = ok && mbar_wait(&mma_done[s], (uint32_t)((i >> 1) & 1), g.err);
      tc_fence_after();
      __syncwarp();
      bool m = row_ok && t >= sh;
      if (g.mask && m) m = g.mask[((size_t)b * g.T + t) * g.mask_L + l] != 0;
      const uint32_t lq = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(s * 128);
      uint32_t dv[32];  // dh, then dx (bits), then the dW^T row: one buffer
      tmem_ld32(lq + half * 32, dv);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float r0 = __uint_as_float(rx[e] << 16), r1 = __uint_as_float(rx[e] & 0xffff0000u);
        const float x0 = __uint_as_float(dv[2 * e]) * 2.f * r0;
        const float x1 = __uint_as_float(dv[2 * e + 1]) * 2.f * r1;
        dacc[2 * e] += x0;
        dacc[2 * e + 1] += x1;
        dv[2 * e] = __float_as_uint(x0);
        dv[2 * e + 1] = __float_as_uint(x1);
      }
      const int col = kc * kGbK + half * 32;
      if (ok && m) {
        float* dst = g.dB + ((size_t)b * g.T + (t - sh)) * g.gh + col;
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          gb_red4(dst + e, __uint_as_float(dv[e]), __uint_as_float(dv[e + 1]),
                  __uint_as_float(dv[e + 2]), __uint_as_float(dv[e + 3]));
      }
      // dW_l^T rows j = TMEM lanes 0..3H-1 (quadrants 0 and 1)
      if (q <= 1) {
        tmem_ld32(lq + 64 + half * 32, dv);
        tmem_ld_wait();
        const int j = r;  // q * 32 + lane
        if (ok && j < H3) {
          const int xx = j / H, hh = j - xx * H;
          float* dw = (xx == 0 ? g.dWi : (xx == 1 ? g.dWf : g.dWr)) + ((size_t)l * H + hh) * g.gh + col;
#pragma unroll
          for (int e = 0; e < 32; e += 4)
            gb_red4(dw + e, __uint_as_float(dv[e]), __uint_as_float(dv[e + 1]),
                    __uint_as_float(dv[e + 2]), __uint_as_float(dv[e + 3]));
        }
      }
      tc_fence_before();
      if (l == nl - 1) {  // dA of this slice is complete: only this CTA owns these rows
        if (ok && row_ok) {
          float4* dst = reinterpret_cast<float4*>(g.dA + ((size_t)b * g.T + t) * g.gh + col);
#pragma unroll
          for (int e = 0; e < 8; ++e)
            dst[e] = make_float4(dacc[4 * e], dacc[4 * e + 1], dacc[4 * e + 2], dacc[4 * e + 3]);
        }
#pragma unroll
        for (int e = 0; e < 32; ++e) dacc[e] = 0.f;
      }
    };

    for (int i = 0; i < iters; i += 2) {
      build(i, rx0);
      if (i >= 1) epilogue(i - 1, rx1);
      if (i + 1 < iters) {
        build(i + 1, rx1);
        epilogue(i, rx0);
      }
    }
    if (iters > 0) {
      if ((iters - 1) & 1) epilogue(iters - 1, rx1);
      else epilogue(iters - 1, rx0);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kGbTmemCols);
  }
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" int dh_gate_preacts_bwd(const void* a, int lda, const void* bsrc, int ldb,
                                   const void* wt, const uint8_t* mask, int mask_L, int batch,
                                   int T, int H, int n_lv, int gh, const void* dpi,
                                   const void* dpf, const void* dpr, float* dA, float* dB,
                                   float* dWi, float* dWf, float* dWr, float* dbi, float* dbf,
                                   float* dbr, int* status, void* stream) {
  DH_REQUIRE(a && bsrc && wt && dpi && dpf && dpr && dA && dB && dWi && dWf && dWr && dbi && dbf &&
                 dbr,
             DH_ERR_ARG, "dh_gate_preacts_bwd: null pointer");
  DH_REQUIRE(batch > 0 && T > 0 && n_lv > 0 && n_lv <= 16 && gh % kGbK == 0 && 3 * H <= 48 &&
                 H > 0 && lda % 8 == 0 && ldb % 8 == 0,
             DH_ERR_SHAPE,
             "dh_gate_preacts_bwd: batch=%d T=%d H=%d n_lv=%d gh=%d (gh %% 64 == 0, 3H <= 48)",
             batch, T, H, n_lv, gh);
  DH_REQUIRE(!mask || mask_L >= n_lv, DH_ERR_SHAPE, "dh_gate_preacts_bwd: mask_L < n_lv");
  DH_REQUIRE(aligned16(dpi) && aligned16(dpf) && aligned16(dpr) && aligned16(dA) &&
                 aligned16(dB) && aligned16(dWi) && aligned16(dWf) && aligned16(dWr),
             DH_ERR_ARG, "dh_gate_preacts_bwd: dP and gradient buffers must be 16-byte aligned");
  CUtensorMap ta, tb, tw, tdi, tdf, tdr;
  const uint64_t da[3] = {(uint64_t)gh, (uint64_t)T, (uint64_t)batch};
  const uint64_t sa[2] = {(uint64_t)lda * 2, (uint64_t)lda * 2 * T};
  const uint64_t sb[2] = {(uint64_t)ldb * 2, (uint64_t)ldb * 2 * T};
  const uint32_t box3[3] = {kGbK, kGbT, 1};
  int rc = make_tmap_bf16(&ta, a, 3, da, sa, box3, true);
  if (rc) return rc;
  rc = make_tmap_bf16(&tb, bsrc, 3, da, sb, box3, true);
  if (rc) return rc;
  const uint64_t dw[2] = {(uint64_t)kGbJ, (uint64_t)n_lv * gh};
  const uint64_t sw[1] = {(uint64_t)kGbJ * 2};
  const uint32_t bw[2] = {kGbJ, kGbK};
  rc = make_tmap_bf16(&tw, wt, 2, dw, sw, bw, true);
  if (rc) return rc;
  if (H == 16) {  // dP (batch, T, n_lv, 16): one 32-byte row per (position, level)
    const uint64_t dd[4] = {16, (uint64_t)n_lv, (uint64_t)T, (uint64_t)batch};
    const uint64_t sd[3] = {32, (uint64_t)n_lv * 32, (uint64_t)n_lv * 32 * T};
    const uint32_t bd[4] = {16, 1, kGbT, 1};
    rc = make_tmap_bf16(&tdi, dpi, 4, dd, sd, bd, false);
    if (!rc) rc = make_tmap_bf16(&tdf, dpf, 4, dd, sd, bd, false);
    if (!rc) rc = make_tmap_bf16(&tdr, dpr, 4, dd, sd, bd, false);
    if (rc) return rc;
  } else {  // not read by the kernel at other head counts
    tdi = tdf = tdr = tw;
  }
  GbArgs g{batch, T, H, n_lv, gh, mask_L, mask,
           reinterpret_cast<const __nv_bfloat16*>(dpi), reinterpret_cast<const __nv_bfloat16*>(dpf),
           reinterpret_cast<const __nv_bfloat16*>(dpr), dA, dB, dWi, dWf, dWr, dbi, dbf, dbr,
           status};
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(gate_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGbSmem);
    configured_dev = dev;
  }
  dim3 grid((T + kGbT - 1) / kGbT, batch);
  gate_bwd_kernel<<<grid, kGbThreads, kGbSmem, reinterpret_cast<cudaStream_t>(stream)>>>(
      ta, tb, tw, tdi, tdf, tdr, g);
  return check_launch("gate_bwd_kernel");
}

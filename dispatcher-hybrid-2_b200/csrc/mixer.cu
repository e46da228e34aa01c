// Parallel-forward mixer: tree mask, gate readout on the tensor cores, and
// the dyadic level sweep.
//
// Gate readout (replaces fused_gates.py:38-93 and the einsums of
// modeling_dispatcher.py:100-109).  One CTA owns 128 positions of one
// sequence.  For every 64-wide slice k of the gate-hidden width and every
// level l, a group of four builder warps forms the hidden tile
//      H[t, k] = relu(A[t, k] + m(t, l) * B[t - 2^l, k])^2          (bf16)
// directly in tensor memory (two groups take alternate tiles), and one thread
// issues tcgen05.mma H x W_l^T into a per-level fp32 accumulator in TMEM
// (W_l: the 3H gate rows of level l, padded to NP rows).  The (T, L, gh)
// hidden tensor never exists in HBM.  Shifted B rows come straight from TMA:
// rows t - 2^l < 0 are out of bounds and arrive as zeros, which is exactly
// the wrap mask.  The epilogue adds the bias, applies sigmoid and the
// wrap/doc masks, and writes
//   mode 0: gates (B, H, L, T, 4) bf16 — (admit*m, forget*m + (1-m), transmit, 0)
//   mode 1: pre-activations (B, T, n_lv, H) x 3 bf16 (the reference op)
// and optionally the transmit gates of every level into a decoder rg_hist.
//
// Level sweep (modeling_dispatcher.py:116-120): one CTA per (sequence, head,
// 8-channel slice) keeps the slice of V for all positions in registers (bf16)
// and exchanges the messages by warp shuffles, within each thread or through
// shared memory, depending on the shift.
#include "common.cuh"
#include "tma.cuh"

namespace dh {
namespace {

// ------------------------------------------------------------------ mask
// mask[b, t, l] = (2^l < T) && t >= 2^l && (!doc_reset || doc(t) == doc(t - 2^l)),
// doc(t) = number of EOT tokens strictly before t (modeling_dispatcher.py:282-323).
__global__ void __launch_bounds__(1024) tree_mask_kernel(const int64_t* ids, int T, int L,
                                                         int64_t eot, int doc_reset,
                                                         uint8_t* mask) {
  extern __shared__ int sdoc[];  // [T]
  __shared__ int warp_tot[32];
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int per = (T + 1023) / 1024;
  const int s0 = tid * per;
  int cnt = 0;
  for (int i = 0; i < per; ++i) {
    const int t = s0 + i;
    if (t < T && doc_reset && ids[(size_t)b * T + t] == eot) ++cnt;
  }
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    warp_tot[lane] = v;  // inclusive over warps
  }
  __syncthreads();
  int run = incl - cnt + (warp > 0 ? warp_tot[warp - 1] : 0);  // exclusive prefix
  for (int i = 0; i < per; ++i) {
    const int t = s0 + i;
    if (t < T) {
      sdoc[t] = run;
      if (doc_reset && ids[(size_t)b * T + t] == eot) ++run;
    }
  }
  __syncthreads();
  for (int i = tid; i < T * L; i += blockDim.x) {
    const int t = i / L, l = i - t * L;
    const int s = 1 << l;
    uint8_t m = (s < T && t >= s) ? 1 : 0;
    if (m && doc_reset) m = sdoc[t] == sdoc[t - s];
    mask[(size_t)b * T * L + i] = m;
  }
}

// ------------------------------------------------------------------ gates
// One CTA per 128 positions of one sequence.  For every 64-column slice of the
// gate-hidden width the CTA builds relu^2(A + m*B[t - 2^l]) for each level
// straight into tensor memory and contracts it with W_l on the tensor cores
// (A operand from TMEM, W from shared memory; accumulators in TMEM, one
// NP-column block per level).  TMEM holds the accumulators of one group of
// levels in columns [0, 384) and four hidden tiles in [384, 512).  Levels are
// processed in groups that fit:
//   group 0, levels 0..min(8, 384/NP)-1 (shift <= 128): one 256-row B window
//            [t0-128, t0+128) loaded together with the A tile serves them all;
//   later groups: B tiles of 128 rows, two levels per stage.
// W is loaded four levels (4*NP rows) per copy.  Fewer, larger copies keep
// the TMA queue short: each copy costs the pipeline a roughly fixed amount of
// time whatever its size.
constexpr int kTileT = 128;
constexpr int kSlice = 64;                    // gate-hidden columns per step (128 B of bf16)
constexpr int kSBytes = kTileT * kSlice * 2;  // 16 KB operand tile
constexpr int kWinLevels = 8;                 // levels served by the B window (2^l <= kTileT)
constexpr int kABStages = 2;                  // A + B-region stages
constexpr int kABBytes = 3 * kSBytes;         // A tile + 32 KB B region (window or two tiles)
constexpr int kWLevels = 4;                   // levels of W per copy
constexpr int kBuilderWarps = 8;              // 2 threads per tile row
constexpr int kGateWaiterWarp = 2 + kBuilderWarps;  // mbarrier waits for the MMA warp
constexpr int kGateThreads = 64 + kBuilderWarps * 32 + 32;
constexpr int kGateHandoffBar = 4;                    // named barrier: MMA warp + waiter warp

// Named barrier of the MMA and waiter warps that also ANDs a flag across them
// (all 64 threads, once per hidden tile, in lockstep).  The MMA warp never
// waits on an mbarrier itself: on B200 an mbarrier wait in the issuing thread
// stalls the tensor pipe (a satisfied try_wait per four MMAs nearly triples
// their time), a named barrier does not.
__device__ __forceinline__ bool gate_handoff(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 64, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "n"(kGateHandoffBar)
      : "memory");
  return r != 0;
}
constexpr int kHBufs = 4;                     // hidden tiles in flight (TMEM)
constexpr int kHCols = kSlice / 2;            // TMEM columns of one hidden tile (2 bf16 each)
constexpr int kHCol0 = 512 - kHBufs * kHCols; // first hidden-tile column
constexpr int kBiasMax = 16 * 64;             // L * NP floats
constexpr int kMaxWStages = 3;

struct GateArgs {
  int B, T, H, L, NP, gh;
  int n_lv, n_calc;
  int nws;            // W stages (3 when NP <= 48, else 2)
  const float* bias;  // (L, NP)
  const uint8_t* mask;
  int mask_L;
  int mode;
  __nv_bfloat16* gates;
  __nv_bfloat16 *pre_i, *pre_f, *pre_r;
  __nv_bfloat16* rg_hist;
  int rg_T;
  int* err;
  uint32_t wait_limit;  // polls of each bounded wait before it reports a timeout
};

__host__ __device__ constexpr int gate_wbytes(int NP) { return kWLevels * NP * 128; }
__host__ __device__ constexpr int gate_smem(int NP, int nws) {
  return 1024 + kABStages * kABBytes + nws * gate_wbytes(NP) + 2 * kSBytes + kBiasMax * 4 + 256;
}

// level groups: group 0 = the window levels, then groups of `cap` levels,
// cap = accumulator blocks that fit in front of the hidden tiles
__device__ __forceinline__ int gate_cap(int NP) { return kHCol0 / NP; }
__device__ __forceinline__ int gate_g0(int NP) { return min(gate_cap(NP), kWinLevels); }
__device__ __forceinline__ int gate_ngroups(int n_calc, int NP) {
  const int g0 = gate_g0(NP), cap = gate_cap(NP);
  return n_calc <= g0 ? 1 : 1 + (n_calc - g0 + cap - 1) / cap;
}
__device__ __forceinline__ void gate_group(int grp, int n_calc, int NP, int& l0, int& l1) {
  const int g0 = gate_g0(NP), cap = gate_cap(NP);
  l0 = grp == 0 ? 0 : g0 + (grp - 1) * cap;
  l1 = min(grp == 0 ? g0 : l0 + cap, n_calc);
}
// AB stages of a group for one slice, and the levels each one serves
__device__ __forceinline__ int gate_nab(int grp, int l0, int l1) {
  return grp == 0 ? 1 : (l1 - l0 + 1) / 2;
}
__device__ __forceinline__ void gate_ab_levels(int grp, int i, int l0, int l1, int& a0, int& a1) {
  if (grp == 0) {
    a0 = l0;
    a1 = l1;
  } else {
    a0 = l0 + 2 * i;
    a1 = min(a0 + 2, l1);
  }
}

__global__ void __launch_bounds__(kGateThreads, 1)
    gate_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmBw, const __grid_constant__ CUtensorMap tmW,
                GateArgs g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int wbytes = gate_wbytes(g.NP);
  uint8_t* sAB = smem;                                  // kABStages x (A 16 KB + B 32 KB)
  uint8_t* sW = sAB + kABStages * kABBytes;             // nws x (4 * NP rows of 128 B)
  uint8_t* sStg = sW + g.nws * wbytes;                  // 2 x 16 KB epilogue staging
  float* sBias = reinterpret_cast<float*>(sStg + 2 * kSBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sBias + kBiasMax);
  uint64_t* ab_full = bars;
  uint64_t* ab_empty = ab_full + kABStages;
  uint64_t* w_full = ab_empty + kABStages;
  uint64_t* w_empty = w_full + kMaxWStages;
  uint64_t* h_full = w_empty + kMaxWStages;
  uint64_t* h_empty = h_full + kHBufs;
  uint64_t* d_full = h_empty + kHBufs;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(d_full + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * kTileT, b = blockIdx.y;
  const int nk = g.gh / kSlice;
  const int ngroups = gate_ngroups(g.n_calc, g.NP);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kABStages; ++i) {
      mbar_init(&ab_full[i], 1);
      mbar_init(&ab_empty[i], kBuilderWarps);
    }
    for (int i = 0; i < g.nws; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], 1);
    }
    for (int i = 0; i < kHBufs; ++i) {
      mbar_init(&h_full[i], kBuilderWarps / 2);  // one builder group per tile
      mbar_init(&h_empty[i], 1);
    }
    mbar_init(d_full, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmBw);
    prefetch_tmap(&tmW);
  }
  for (int i = threadIdx.x; i < g.L * g.NP; i += blockDim.x) sBias[i] = g.bias[i];
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int abs_ = 0, ws = 0;
      uint32_t abph = 0, wph = 0;
      long fills_ab = 0, fills_w = 0;
      bool ok = true;
      for (int grp = 0; grp < ngroups && ok; ++grp) {
        int l0, l1;
        gate_group(grp, g.n_calc, g.NP, l0, l1);
        const int nab = gate_nab(grp, l0, l1);
        for (int kc = 0; kc < nk && ok; ++kc) {
          const int x = kc * kSlice;
          // W of the group's levels, kWLevels levels per copy
          for (int c0 = l0; c0 < l1 && ok; c0 += kWLevels) {
            if (!mbar_wait(&w_empty[ws], wph ^ 1, g.err, g.wait_limit)) { ok = false; break; }
            mbar_arrive_expect_tx(&w_full[ws], (uint32_t)wbytes);
            tma_load_2d(&tmW, &w_full[ws], sW + ws * wbytes, x, c0 * g.NP);
            ++fills_w;
            if (++ws == g.nws) { ws = 0; wph ^= 1; }
          }
          // A tile + the B rows of the stage's levels
          for (int i = 0; i < nab && ok; ++i) {
            if (!mbar_wait(&ab_empty[abs_], abph ^ 1, g.err, g.wait_limit)) { ok = false; break; }
            uint8_t* st = sAB + abs_ * kABBytes;
            int a0, a1;
            gate_ab_levels(grp, i, l0, l1, a0, a1);
            const uint32_t bytes = grp == 0 ? 3u * kSBytes : (uint32_t)(1 + a1 - a0) * kSBytes;
            mbar_arrive_expect_tx(&ab_full[abs_], bytes);
            tma_load_3d(&tmA, &ab_full[abs_], st, x, t0, b);
            if (grp == 0) {
              // window rows [t0 - 128, t0 + 128); rows before 0 arrive as zeros
              tma_load_3d(&tmBw, &ab_full[abs_], st + kSBytes, x, t0 - kTileT, b);
            } else {
              for (int l = a0; l < a1; ++l)
                tma_load_3d(&tmB, &ab_full[abs_], st + (1 + l - a0) * kSBytes, x, t0 - (1 << l), b);
            }
            ++fills_ab;
            if (++abs_ == kABStages) { abs_ = 0; abph ^= 1; }
          }
        }
      }
      // drain: no copy may still be writing shared memory when the CTA exits
      for (int i = 0; i < kABStages; ++i) {
        const long n = fills_ab / kABStages + (i < fills_ab % kABStages ? 1 : 0);
        if (n > 0) mbar_wait(&ab_full[i], (uint32_t)((n - 1) & 1), nullptr, 1u << 20);
      }
      for (int i = 0; i < g.nws; ++i) {
        const long n = fills_w / g.nws + (i < fills_w % g.nws ? 1 : 0);
        if (n > 0) mbar_wait(&w_full[i], (uint32_t)((n - 1) & 1), nullptr, 1u << 20);
      }
    }
  } else if (warp == 1) {  // ---------------- MMA issue (no mbarrier waits here)
    const uint32_t idesc = idesc_bf16(kTileT, g.NP);
    int ws = 0, hs = 0;
    bool ok = true;
    for (int grp = 0; grp < ngroups; ++grp) {
      int l0, l1;
      gate_group(grp, g.n_calc, g.NP, l0, l1);
      for (int kc = 0; kc < nk; ++kc) {
        for (int l = l0; l < l1; ++l) {
          const int c0 = l0 + ((l - l0) / kWLevels) * kWLevels;
          ok = gate_handoff(ok);  // the waiter saw this tile built (and its W copy landed)
          tc_fence_after();
          if (ok && lane == 0) {
            const uint32_t hA = tmem_base + (uint32_t)(kHCol0 + hs * kHCols);
            const uint32_t wB = smem_u32(sW + ws * wbytes + (l - c0) * g.NP * 128);
            const uint32_t d = tmem_base + (uint32_t)((l - l0) * g.NP);
#pragma unroll
            for (int k = 0; k < kSlice / 16; ++k)  // 16 bf16 of K = 8 TMEM columns
              umma_bf16_ts(d, hA + k * 8, sw128_desc(wB + k * 32), idesc, (kc | k) != 0);
            umma_commit(&h_empty[hs]);
          }
          if (++hs == kHBufs) hs = 0;
          if (l + 1 == l1 || l + 1 == c0 + kWLevels) {  // last level of this W copy
            if (ok && lane == 0) umma_commit(&w_empty[ws]);
            if (++ws == g.nws) ws = 0;
          }
          __syncwarp();
        }
      }
      if (ok && lane == 0) umma_commit(d_full);
      __syncwarp();
    }
  } else if (warp == kGateWaiterWarp) {  // ---------------- waiter for the MMA warp
    int ws = 0, hs = 0;
    uint32_t wph = 0, hph = 0;
    bool ok = true;
    for (int grp = 0; grp < ngroups; ++grp) {
      int l0, l1;
      gate_group(grp, g.n_calc, g.NP, l0, l1);
      for (int kc = 0; kc < nk; ++kc) {
        for (int l = l0; l < l1; ++l) {
          const int c0 = l0 + ((l - l0) / kWLevels) * kWLevels;
          // after a failed (bounded) wait, skip every later wait but keep the
          // handoffs, so the two warps stay in lockstep and nothing blocks
          if (l == c0) ok = ok && mbar_wait(&w_full[ws], wph, g.err, g.wait_limit);
          ok = ok && mbar_wait(&h_full[hs], hph, g.err, g.wait_limit);
          ok = gate_handoff(ok);
          if (++hs == kHBufs) { hs = 0; hph ^= 1; }
          if (l + 1 == l1 || l + 1 == c0 + kWLevels) {
            if (++ws == g.nws) { ws = 0; wph ^= 1; }
          }
        }
      }
    }
  } else {  // ---------------- builders + epilogue (warps 2..9)
    const int q = warp & 3;               // TMEM lane quadrant of this warp
    const int half = (warp - 2) >> 2;     // builder group: alternate hidden tiles / epilogue levels
    const int r = q * 32 + lane;          // tile row == TMEM lane
    const int t = t0 + r;
    const bool row_ok = t < g.T;
    // per-level mask bits of this row, read once (wrap + doc reset)
    uint32_t mbits = 0;
    for (int l = 0; l < g.n_calc; ++l) {
      bool m = t >= (1 << l);
      if (g.mask) m = row_ok && g.mask[((size_t)b * g.T + t) * g.mask_L + l] != 0;
      mbits |= (m ? 1u : 0u) << l;
    }
    int abs_ = 0, hs = 0, jt = 0;  // jt: hidden tiles so far (same count in every thread)
    uint32_t abph = 0, hph = 0, dph = 0;
    // A failed (bounded) wait clears `ok`; the thread then skips every
    // further wait but still walks the same loops, so each named barrier
    // below is reached by all builder threads and nothing can hang.
    bool ok = true;
    for (int grp = 0; grp < ngroups; ++grp) {
      int l0, l1;
      gate_group(grp, g.n_calc, g.NP, l0, l1);
      const int nab = gate_nab(grp, l0, l1);
      for (int kc = 0; kc < nk; ++kc) {
        for (int i = 0; i < nab; ++i) {
          ok = ok && mbar_wait(&ab_full[abs_], abph, g.err, g.wait_limit);
          const uint8_t* st = sAB + abs_ * kABBytes;
          uint4 av[8];  // this row of the A slice (64 columns)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            av[j] = *reinterpret_cast<const uint4*>(st + r * 128 + ((j ^ (r & 7)) << 4));
          int a0, a1;
          gate_ab_levels(grp, i, l0, l1, a0, a1);
          for (int l = a0; l < a1; ++l, ++jt) {
            // the two builder groups (warps 2-5, 6-9) take alternate tiles, so
            // two tiles are in flight; each thread builds one whole row
            if ((jt & 1) == half) {
              ok = ok && mbar_wait(&h_empty[hs], hph ^ 1, g.err, g.wait_limit);
              tc_fence_after();
              // source row t - 2^l: row r + 128 - 2^l of the window (group 0) or
              // row r of the level's own tile (group 1); rows before position 0
              // arrive as TMA zeros, which is the wrap mask
              const int bi = grp == 0 ? r + kTileT - (1 << l) : r;
              const uint8_t* brow =
                  st + (grp == 0 ? kSBytes : (1 + l - a0) * kSBytes) + bi * 128;
              // masked rows drop the shifted source
              const float mf = g.mask ? (float)((mbits >> l) & 1u) : 1.f;
              const __nv_bfloat162 m2 = __floats2bfloat162_rn(mf, mf);
              const __nv_bfloat162 z2 = __floats2bfloat162_rn(0.f, 0.f);
              uint32_t hv[32];  // this row's 64 hidden values, two per TMEM column
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                uint4 bv = *reinterpret_cast<const uint4*>(brow + ((j ^ (bi & 7)) << 4));
                const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&av[j]);
                __nv_bfloat162* b2 = reinterpret_cast<__nv_bfloat162*>(&bv);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  // bf16 arithmetic as in the reference: (A + m*B) rounded once, relu, squared
                  __nv_bfloat162 x = __hfma2(m2, b2[e], a2[e]);
                  x = __hmax2(x, z2);
                  b2[e] = __hmul2_rn(x, x);
                }
                hv[4 * j] = bv.x;
                hv[4 * j + 1] = bv.y;
                hv[4 * j + 2] = bv.z;
                hv[4 * j + 3] = bv.w;
              }
              tmem_st32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(kHCol0 + hs * kHCols),
                        hv);
              tmem_st_wait();
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&h_full[hs]);
            }
            if (++hs == kHBufs) { hs = 0; hph ^= 1; }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&ab_empty[abs_]);
          if (++abs_ == kABStages) { abs_ = 0; abph ^= 1; }
        }
      }
      // ---- epilogue of this level group: the two warp halves split the levels.
      // All MMAs of the group are complete: half k stages each level's
      // (3H x 128) gate tile in staging buffer k, column-major, and the half
      // then writes it as 16-byte runs along T.
      ok = ok && mbar_wait(d_full, dph, g.err, g.wait_limit);
      dph ^= 1;
      tc_fence_after();
      const int H = g.H;
      const int nl = l1 - l0, mid = (nl + 1) / 2;
      const int la = half ? l0 + mid : l0, lb = half ? l1 : l0 + mid;
      __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(sStg + half * kSBytes);
      for (int l = la; l < lb; ++l) {
        const uint32_t base = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)((l - l0) * g.NP);
        const float* bias = sBias + l * g.NP;
        const float m = (float)((mbits >> l) & 1u);
        const int H3 = 3 * H;
        const bool mode0 = g.mode == 0;
        if (mode0 && H == 16) {
          // 16 heads: the three 16-column chunks are the admit, forget and
          // transmit gates; each thread writes its own position's (a, f, r, 0)
          // per head, straight from registers (consecutive lanes are
          // consecutive positions, so a warp's 8-byte stores form one
          // contiguous run): no staging and no barriers
          uint32_t pk[3][8];
#pragma unroll
          for (int c = 0; c < 3; ++c) {
            uint32_t v[16];
            tmem_ld16(base + c * 16, v);
            tmem_ld_wait();
            float sg[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) sg[e] = sigmoidf_(__uint_as_float(v[e]) + bias[c * 16 + e]);
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              float x0 = sg[e], x1 = sg[e + 1];
              if (c == 0) {
                x0 *= m;
                x1 *= m;
              } else if (c == 1) {
                x0 = fmaf(x0, m, 1.f - m);
                x1 = fmaf(x1, m, 1.f - m);
              }
              pk[c][e / 2] = pack2(x0, x1);
            }
            if (c == 2 && g.rg_hist && row_ok) {  // transmit gates into the decoder cache
              __nv_bfloat16* rg = g.rg_hist + (((size_t)b * g.rg_T + t) * g.L + l) * 16;
#pragma unroll
              for (int e = 0; e < 16; ++e) rg[e] = f2bf(sg[e]);
            }
          }
          if (l < g.n_lv && row_ok) {
#pragma unroll
            for (int hh = 0; hh < 16; ++hh) {
              const int sh = (hh & 1) * 16;
              const uint32_t ga = (pk[0][hh >> 1] >> sh) & 0xffffu;
              const uint32_t gf = (pk[1][hh >> 1] >> sh) & 0xffffu;
              const uint32_t gr = (pk[2][hh >> 1] >> sh) & 0xffffu;
              *reinterpret_cast<uint2*>(g.gates + ((((size_t)b * 16 + hh) * g.L + l) * g.T + t) * 4) =
                  make_uint2(ga | (gf << 16), gr);
            }
          }
          continue;
        }
        for (int c = 0; c < H3; c += 16) {
          uint32_t v[16];
          tmem_ld16(base + c, v);
          tmem_ld_wait();
          // 16 independent columns with no early exit and no division, so the
          // exp / reciprocal chains of the columns overlap.  Columns past 3H
          // are the zero padding up to NP (bias 0): computed, never stored.
          float val[16], sg[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const int col = c + e;
            const float pre = __uint_as_float(v[e]) + bias[col];
            sg[e] = sigmoidf_(pre);
            const float gated = col < H ? sg[e] * m : (col < 2 * H ? fmaf(sg[e], m, 1.f - m) : sg[e]);
            val[e] = mode0 ? gated : pre;
          }
#pragma unroll
          for (int e = 0; e < 16; ++e)
            if (c + e < H3) stg[(c + e) * kTileT + r] = f2bf(val[e]);
          if (g.rg_hist && row_ok) {  // transmit gates (columns 2H..3H-1) into the decoder cache
            __nv_bfloat16* rg = g.rg_hist + (((size_t)b * g.rg_T + t) * g.L + l) * H;
#pragma unroll
            for (int e = 0; e < 16; ++e)
              if (c + e >= 2 * H && c + e < H3) rg[c + e - 2 * H] = f2bf(sg[e]);
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
        if (l < g.n_lv) {
          const int tid_h = q * 32 + lane;  // 0..127 within this half
          if (g.mode == 0) {
            // gates (B, H, L, T, 4): (admit, forget, transmit, 0) per position,
            // two positions per store; tile column col = gi*H + h
            static_assert(kTileT / 2 == 64, "64 position pairs per tile");
            const int chunks = H * (kTileT / 2);
#pragma unroll 2
            for (int ck = tid_h; ck < chunks; ck += 128) {
              const int h = ck >> 6, p = (ck & 63) * 2;
              const int tt = t0 + p;
              if (tt >= g.T) continue;
              uint32_t w[4];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const uint32_t ga = __bfloat16_as_ushort(stg[h * kTileT + p + e]);
                const uint32_t gf = __bfloat16_as_ushort(stg[(H + h) * kTileT + p + e]);
                const uint32_t gr = __bfloat16_as_ushort(stg[(2 * H + h) * kTileT + p + e]);
                w[2 * e] = ga | (gf << 16);
                w[2 * e + 1] = gr;
              }
              // 8 bytes per position: a pair is 16-byte aligned only when its
              // first position index (over the whole buffer) is even, which
              // fails for odd T on every other (head, level) row
              const size_t e0 = (((size_t)b * H + h) * g.L + l) * (size_t)g.T + tt;
              __nv_bfloat16* dst = g.gates + e0 * 4;
              if (tt + 1 < g.T && (e0 & 1) == 0) {
                *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
              } else {
                *reinterpret_cast<uint2*>(dst) = make_uint2(w[0], w[1]);
                if (tt + 1 < g.T) *reinterpret_cast<uint2*>(dst + 4) = make_uint2(w[2], w[3]);
              }
            }
          } else if (row_ok) {
            const size_t o = (((size_t)b * g.T + t) * g.n_lv + l) * H;
            for (int h = 0; h < H; ++h) {
              g.pre_i[o + h] = stg[h * kTileT + r];
              g.pre_f[o + h] = stg[(H + h) * kTileT + r];
              g.pre_r[o + h] = stg[(2 * H + h) * kTileT + r];
            }
          }
        }
        asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
      }
      // both halves must be done reading this group's accumulators before
      // either builds hidden tiles that start the next group's MMAs
      asm volatile("bar.sync 3, %0;" ::"n"(kBuilderWarps * 32) : "memory");
      tc_fence_before();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

// ------------------------------------------------------------------ scan
// One CTA per (sequence, head, 8-channel slice); warp w owns the 128
// consecutive positions [128 w, 128 w + 128), lane j the positions
// 128 w + 32 i + j (i = 0..3).  Per level l (shift s = 2^l), in the
// reference's order and rounding (modeling_dispatcher.py:116-120, bf16):
//   msg(t) = r(t) * V(t)
//   V(t)   = f(t) * V(t) + a(t) * msg(t - s)
// in bf16x2 arithmetic, one rounding per product and per sum (the _rn forms:
// no multiply-add contraction, as in the reference's separate bf16 ops), so
// the sweep is bit-exact against the reference's loop.  Where msg(t - s)
// comes from depends on s:
//   s < 32      lane j - s of the same warp (a shuffle), for the first s lanes
//               of row 0 the previous warp's row 3 (through shared memory)
//   s = 32, 64  this thread's own row i - s/32, for the first rows the
//               previous warp's last rows (through shared memory)
//   s >= 128    any warp: every message goes through shared memory
// Each level has one barrier; the shared buffer is double buffered by level
// parity (a half is rewritten two levels later, after a barrier every reader
// of it has passed).  Each thread loads only its own positions' gates (one
// 8-byte load per position, coalesced along the warp), a level ahead.
constexpr int kScanThreads = 1024;  // 32 warps hide the per-level barrier latency
constexpr int kScanPer = 4;        // positions per thread (T <= 4096)
constexpr int kScanXch = 2048;     // minimum entries of a buffer half (the small exchanges)

struct ScanArgs {
  const __nv_bfloat16* v0;
  int ld_v0;
  const __nv_bfloat16* gates;  // (B, H, L, T, 4)
  __nv_bfloat16* out;
  int ld_out;
  int B, T, H, hd, L, n_lv;
  __nv_bfloat16* ring;  // (B, S, d) or null
  int S;
};

// position of row i of this thread
__device__ __forceinline__ int scan_pos(int tid, int i) {
  return ((tid >> 5) << 7) + (i << 5) + (tid & 31);
}

struct LevelGates {
  uint2 g[kScanPer];  // (admit | forget << 16, transmit) of each owned position
};

__device__ __forceinline__ void load_level(const __nv_bfloat16* __restrict__ gl, int T, int tid,
                                           LevelGates& G) {
  // Unconditional loads (positions past the end read the last one and are
  // never used): a select on the loaded value would make the thread wait for
  // the loads here instead of where the next level consumes them.
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int t = min(scan_pos(tid, i), T - 1);
    G.g[i] = __ldg(reinterpret_cast<const uint2*>(gl) + t);
  }
}

struct ScanState {
  uint4 V[kScanPer];
};

__device__ __forceinline__ void write_ring(const ScanArgs& a, const ScanState& st, int b, int col,
                                           int tid, int j) {
  const int T = a.T, d = a.H * a.hd;
  const int lo = T - (2 << j);
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int t = scan_pos(tid, i);
    if (t < T && t >= lo) {
      const int slot = ((2 << j) - 2) + (t & ((2 << j) - 1));
      *reinterpret_cast<uint4*>(a.ring + ((size_t)b * a.S + slot) * d + col) = st.V[i];
    }
  }
}

// broadcast the low / high bf16 of a 32-bit word to both halves
__device__ __forceinline__ __nv_bfloat162 bcast_lo(uint32_t w) {
  const uint32_t x = __byte_perm(w, w, 0x1010);
  return *reinterpret_cast<const __nv_bfloat162*>(&x);
}
__device__ __forceinline__ __nv_bfloat162 bcast_hi(uint32_t w) {
  const uint32_t x = __byte_perm(w, w, 0x3232);
  return *reinterpret_cast<const __nv_bfloat162*>(&x);
}

// msg = r * V of one position (8 channels)
__device__ __forceinline__ uint4 scan_msg(const uint4& v, uint32_t gy) {
  const __nv_bfloat162 r2 = bcast_lo(gy);
  uint4 m = v;
  __nv_bfloat162* mv = reinterpret_cast<__nv_bfloat162*>(&m);
#pragma unroll
  for (int e = 0; e < 4; ++e) mv[e] = __hmul2_rn(r2, mv[e]);
  return m;
}

// V = f V + a m  (m = msg(t - s)), or V = f V where no source exists
__device__ __forceinline__ void scan_update(uint4& v4, uint32_t gx, const uint4& m) {
  const __nv_bfloat162 a2 = bcast_lo(gx), f2 = bcast_hi(gx);
  __nv_bfloat162* v = reinterpret_cast<__nv_bfloat162*>(&v4);
  const __nv_bfloat162* mv = reinterpret_cast<const __nv_bfloat162*>(&m);
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = __hadd2_rn(__hmul2_rn(f2, v[e]), __hmul2_rn(a2, mv[e]));
}
__device__ __forceinline__ void scan_forget_only(uint4& v4, uint32_t gx) {
  const __nv_bfloat162 f2 = bcast_hi(gx);
  __nv_bfloat162* v = reinterpret_cast<__nv_bfloat162*>(&v4);
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = __hmul2_rn(f2, v[e]);
}

__device__ __forceinline__ uint4 shfl4(const uint4& m, int src) {
  return make_uint4(__shfl_sync(0xffffffffu, m.x, src), __shfl_sync(0xffffffffu, m.y, src),
                    __shfl_sync(0xffffffffu, m.z, src), __shfl_sync(0xffffffffu, m.w, src));
}

// s < 32: lane j - s of the same warp; lanes j < s take row i - 1 of lane
// j - s + 32, and at row 0 the previous warp's row 3
__device__ __forceinline__ void scan_level_lanes(ScanState& st, const LevelGates& cur, uint4* xb,
                                                 int T, int tid, int s) {
  const int w = tid >> 5, j = tid & 31, src = (j - s) & 31;
  const uint4 m3 = scan_msg(st.V[3], cur.g[3].y);
  xb[w * 32 + j] = m3;
  __syncthreads();
  uint4 rprev = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    // row i's message, taken before row i is updated (rows ascend)
    const uint4 mi = i == kScanPer - 1 ? m3 : scan_msg(st.V[i], cur.g[i].y);
    const uint4 rc = shfl4(mi, src);  // every lane takes part
    const int t = scan_pos(tid, i);
    if (t < T) {
      if (t < s) {
        scan_forget_only(st.V[i], cur.g[i].x);
      } else {
        const uint4 m = j >= s ? rc : (i > 0 ? rprev : xb[(w - 1) * 32 + src]);
        scan_update(st.V[i], cur.g[i].x, m);
      }
    }
    rprev = rc;
  }
}

// s = 32 K (K = 1, 2): row i - K of this thread; rows i < K from the previous
// warp's rows i - K + 4
template <int K>
__device__ __forceinline__ void scan_level_rows(ScanState& st, const LevelGates& cur, uint4* xb,
                                                int T, int tid) {
  const int w = tid >> 5, j = tid & 31;
  uint4 m[kScanPer];
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) m[i] = scan_msg(st.V[i], cur.g[i].y);
#pragma unroll
  for (int q = 0; q < K; ++q) xb[(w * 2 + q) * 32 + j] = m[kScanPer - K + q];
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int t = scan_pos(tid, i);
    if (t >= T) continue;
    if (t < 32 * K) {
      scan_forget_only(st.V[i], cur.g[i].x);
    } else {
      const uint4 mm = i >= K ? m[i >= K ? i - K : 0] : xb[((w - 1) * 2 + i) * 32 + j];
      scan_update(st.V[i], cur.g[i].x, mm);
    }
  }
}

// s >= 128: through shared memory, indexed by position
__device__ __forceinline__ void scan_level_smem(ScanState& st, const LevelGates& cur, uint4* xb,
                                                int T, int tid, int s) {
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int t = scan_pos(tid, i);
    if (t < T) xb[t] = scan_msg(st.V[i], cur.g[i].y);
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int t = scan_pos(tid, i);
    if (t >= T) continue;
    if (t >= s) scan_update(st.V[i], cur.g[i].x, xb[t - s]);
    else scan_forget_only(st.V[i], cur.g[i].x);
  }
}

// one level of the sweep; loads the next level's gates into `nxt` first
__device__ __forceinline__ void scan_level(const ScanArgs& a, ScanState& st, uint4* sx, int half,
                                           const __nv_bfloat16* gbase, int b, int col, int tid,
                                           int l, int nl, const LevelGates& cur,
                                           LevelGates& nxt) {
  const int T = a.T, s = 1 << l;
  if (l + 1 < nl) load_level(gbase + (size_t)(l + 1) * 4 * T, T, tid, nxt);
  uint4* xb = sx + (l & 1) * half;  // this level's half of the message buffer
  if (s < 32) scan_level_lanes(st, cur, xb, T, tid, s);
  else if (s == 32) scan_level_rows<1>(st, cur, xb, T, tid);
  else if (s == 64) scan_level_rows<2>(st, cur, xb, T, tid);
  else scan_level_smem(st, cur, xb, T, tid, s);
  if (a.ring && l + 1 < a.L) write_ring(a, st, b, col, tid, l + 1);
}

__global__ void __launch_bounds__(kScanThreads) scan_kernel(ScanArgs a) {
  extern __shared__ uint4 sx[];  // 2 x [max(T, kScanXch)] x 8 bf16
  const int slices = a.hd / 8;
  const int cc = blockIdx.x % slices;
  const int h = (blockIdx.x / slices) % a.H;
  const int b = blockIdx.x / (slices * a.H);
  const int col = h * a.hd + cc * 8;
  const int tid = threadIdx.x;
  const int T = a.T;
  const int half = T > kScanXch ? T : kScanXch;
  const __nv_bfloat16* gbase = a.gates + (((size_t)b * a.H + h) * a.L) * 4 * (size_t)T;
  int nl = a.n_lv;
  while (nl > 0 && (1 << (nl - 1)) > T) --nl;   // the reference stops at shift > T
  ScanState st;
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int t = scan_pos(tid, i);
    // unconditional load (positions past the end read the last one, never
    // used): a select on the loaded value would stall here
    st.V[i] = *reinterpret_cast<const uint4*>(a.v0 + ((size_t)b * T + min(t, T - 1)) * a.ld_v0 +
                                              col);
  }
  if (a.ring) write_ring(a, st, b, col, tid, 0);
  LevelGates g0, g1;
  if (nl > 0) load_level(gbase, T, tid, g0);
  for (int l = 0; l < nl; l += 2) {
    scan_level(a, st, sx, half, gbase, b, col, tid, l, nl, g0, g1);
    if (l + 1 < nl) scan_level(a, st, sx, half, gbase, b, col, tid, l + 1, nl, g1, g0);
  }
  if (a.ring)
    for (int j = a.n_lv + 1; j < a.L; ++j) write_ring(a, st, b, col, tid, j);
#pragma unroll
  for (int i = 0; i < kScanPer; ++i) {
    const int t = scan_pos(tid, i);
    if (t < T) *reinterpret_cast<uint4*>(a.out + ((size_t)b * T + t) * a.ld_out + col) = st.V[i];
  }
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" int dh_tree_mask(const int64_t* ids, int batch, int T, int L, int64_t eot,
                            int doc_reset, uint8_t* mask, void* stream) {
  DH_REQUIRE(ids && mask, DH_ERR_ARG, "dh_tree_mask: null pointer");
  DH_REQUIRE(batch > 0 && T > 0 && T <= 16384 && L > 0 && L < 31, DH_ERR_SHAPE,
             "dh_tree_mask: bad sizes");
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(tree_mask_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 16384 * 4);
    configured_dev = dev;
  }
  tree_mask_kernel<<<batch, 1024, (size_t)T * sizeof(int), reinterpret_cast<cudaStream_t>(stream)>>>(
      ids, T, L, eot, doc_reset, mask);
  return check_launch("tree_mask_kernel");
}

static int launch_gates(const void* a, int lda, const void* bsrc, int ldb, const void* wg,
                        GateArgs g, cudaStream_t st) {
  DH_REQUIRE(a && bsrc && wg && g.bias, DH_ERR_ARG, "mixer gates: null pointer");
  DH_REQUIRE(g.B > 0 && g.T > 0 && g.H > 0, DH_ERR_SHAPE, "mixer gates: batch=%d T=%d H=%d",
             g.B, g.T, g.H);
  DH_REQUIRE(g.gh % kSlice == 0 && g.NP % 16 == 0 && g.NP <= 64 && 3 * g.H <= g.NP,
             DH_ERR_SHAPE, "mixer gates: gh=%d NP=%d H=%d unsupported", g.gh, g.NP, g.H);
  DH_REQUIRE(g.n_calc >= 1 && g.n_calc <= g.L && g.n_lv <= g.n_calc && g.L * g.NP <= kBiasMax,
             DH_ERR_SHAPE,
             "mixer gates: level counts n_lv=%d n_calc=%d L=%d", g.n_lv, g.n_calc, g.L);
  DH_REQUIRE(lda % 8 == 0 && ldb % 8 == 0, DH_ERR_SHAPE, "mixer gates: row strides must be multiples of 8");
  DH_REQUIRE(!g.mask || g.mask_L >= g.n_calc, DH_ERR_SHAPE,
             "mixer gates: mask has %d levels per position, %d are read", g.mask_L, g.n_calc);
  g.nws = g.NP <= 48 ? 3 : 2;
  g.wait_limit = wait_limit();
  const int smem = gate_smem(g.NP, g.nws);
  CUtensorMap ta, tb, tbw, tw;
  const uint64_t da[3] = {(uint64_t)g.gh, (uint64_t)g.T, (uint64_t)g.B};
  const uint64_t sa[2] = {(uint64_t)lda * 2, (uint64_t)lda * 2 * g.T};
  const uint64_t sb[2] = {(uint64_t)ldb * 2, (uint64_t)ldb * 2 * g.T};
  const uint32_t box3[3] = {kSlice, kTileT, 1};
  const uint32_t boxw3[3] = {kSlice, 2 * kTileT, 1};
  int rc = make_tmap_bf16(&ta, a, 3, da, sa, box3, true);
  if (rc) return rc;
  rc = make_tmap_bf16(&tb, bsrc, 3, da, sb, box3, true);
  if (rc) return rc;
  rc = make_tmap_bf16(&tbw, bsrc, 3, da, sb, boxw3, true);
  if (rc) return rc;
  const uint64_t dw[2] = {(uint64_t)g.gh, (uint64_t)g.L * g.NP};
  const uint64_t sw[1] = {(uint64_t)g.gh * 2};
  const uint32_t bw[2] = {kSlice, (uint32_t)(kWLevels * g.NP)};
  rc = make_tmap_bf16(&tw, wg, 2, dw, sw, bw, true);
  if (rc) return rc;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(gate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         gate_smem(64, 2) > gate_smem(48, 3) ? gate_smem(64, 2) : gate_smem(48, 3));
    configured_dev = dev;
  }
  dim3 grid((g.T + kTileT - 1) / kTileT, g.B);
  gate_kernel<<<grid, kGateThreads, smem, st>>>(ta, tb, tbw, tw, g);
  return check_launch("gate_kernel");
}

extern "C" int dh_mixer_gates(const void* a, int lda, const void* bsrc, int ldb, const void* wg,
                              const float* bias, const uint8_t* mask, int batch, int T, int H,
                              int L, int NP, int gh, int n_lv, void* gates, void* rg_hist,
                              int rg_T, int* status, void* stream) {
  DH_REQUIRE(gates, DH_ERR_ARG, "dh_mixer_gates: null gates output");
  GateArgs g{};
  g.B = batch; g.T = T; g.H = H; g.L = L; g.NP = NP; g.gh = gh;
  g.n_lv = n_lv;
  g.n_calc = rg_hist ? L : n_lv;
  g.bias = bias; g.mask = mask; g.mask_L = L; g.mode = 0;
  g.gates = reinterpret_cast<__nv_bfloat16*>(gates);
  g.rg_hist = reinterpret_cast<__nv_bfloat16*>(rg_hist);
  g.rg_T = rg_T;
  g.err = status;
  return launch_gates(a, lda, bsrc, ldb, wg, g, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dh_gate_preacts_fwd(const void* a, int lda, const void* bsrc, int ldb,
                                   const void* wg, const float* bias, const uint8_t* mask,
                                   int mask_L, int batch, int T, int H, int L, int NP, int gh,
                                   int n_lv, void* pre_i, void* pre_f, void* pre_r, int* status,
                                   void* stream) {
  DH_REQUIRE(pre_i && pre_f && pre_r, DH_ERR_ARG, "dh_gate_preacts_fwd: null output");
  GateArgs g{};
  g.B = batch; g.T = T; g.H = H; g.L = L; g.NP = NP; g.gh = gh;
  g.n_lv = n_lv; g.n_calc = n_lv;
  g.bias = bias; g.mask = mask; g.mask_L = mask_L; g.mode = 1;
  g.pre_i = reinterpret_cast<__nv_bfloat16*>(pre_i);
  g.pre_f = reinterpret_cast<__nv_bfloat16*>(pre_f);
  g.pre_r = reinterpret_cast<__nv_bfloat16*>(pre_r);
  g.err = status;
  return launch_gates(a, lda, bsrc, ldb, wg, g, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dh_level_scan(const void* v0, int ld_v0, const void* gates, void* out, int ld_out,
                             int batch, int T, int H, int hd, int L, int n_lv, void* ring,
                             void* stream) {
  DH_REQUIRE(v0 && gates && out, DH_ERR_ARG, "dh_level_scan: null pointer");
  DH_REQUIRE(T > 0 && T <= kScanThreads * kScanPer, DH_ERR_SHAPE,
             "dh_level_scan: T=%d exceeds %d", T, kScanThreads * kScanPer);
  DH_REQUIRE(batch > 0 && H > 0 && hd > 0 && hd % 8 == 0 && ld_v0 % 8 == 0 && ld_out % 8 == 0 &&
                 L >= 1 && L < 30 && n_lv >= 0 && n_lv <= L,
             DH_ERR_SHAPE, "dh_level_scan: bad sizes");
  ScanArgs a{reinterpret_cast<const __nv_bfloat16*>(v0), ld_v0,
             reinterpret_cast<const __nv_bfloat16*>(gates),
             reinterpret_cast<__nv_bfloat16*>(out), ld_out, batch, T, H, hd, L, n_lv,
             reinterpret_cast<__nv_bfloat16*>(ring), (1 << (L + 1)) - 2};
  const int blocks = batch * H * (hd / 8);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         2 * kScanThreads * kScanPer * 16);
    configured_dev = dev;
  }
  const size_t half = (size_t)(T > kScanXch ? T : kScanXch);
  scan_kernel<<<blocks, kScanThreads, half * 32, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("scan_kernel");
}

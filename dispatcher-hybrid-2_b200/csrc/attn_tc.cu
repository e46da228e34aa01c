// Sliding-window causal attention for the parallel forward on the 5th-gen
// tensor cores (modeling_dispatcher.py:168-185: keys s with t - window < s <= t,
// scale 1/sqrt(hd); plain causal when the window covers the sequence).
//
// One CTA per (sequence, head, 128 queries), warp-specialised:
//   warp 4      TMA: Q once, then K and V blocks of 128 keys into a 2-stage ring
//   warp 5      TMEM allocation and one thread issuing tcgen05.mma:
//                 S = Q K^T   (M=128 queries, N=128 keys, K=64)  -> TMEM
//                 O += P V    (A = P from TMEM, B = V read MN-major from its
//                              key-major tile, M=128, N=64, K=128) -> TMEM
//   warps 0-3   one query row per thread (= TMEM lane): mask, online softmax
//               in fp32 (base 2) in two passes over S in TMEM (row maximum,
//               then P as bf16 into TMEM 32 keys at a time, so a thread holds
//               no whole row), rescale O in TMEM when the row's base moves
//               (only when a score passes it by more than 2^8);
//               blocks wholly inside the band skip the mask; final O / l.
// TMEM per CTA: S 128 columns + P 64 + O 64 = 256, and few enough registers
// that two CTAs share an SM: one's softmax overlaps the other's MMAs.  Every
// wait is bounded; a wait that gives up sets *status and the CTA drains.
#include <math.h>

#include "common.cuh"
#include "tma.cuh"

namespace dh {
namespace {

constexpr int kAtHd = 64;
constexpr int kAtBq = 128;
constexpr int kAtBk = 128;
constexpr int kAtTile = 128 * 64 * 2;  // 16 KB: 128 rows of 64 bf16
constexpr int kAtStages = 2;
constexpr int kAtThreads = 192;
constexpr int kAtS = 0, kAtP = 128, kAtO = 192, kAtCols = 256;  // TMEM columns
constexpr int kAtSmem = 1024 + kAtTile + kAtStages * 2 * kAtTile + 256;

struct AtArgs {
  int T, H, window, ldo;
  __nv_bfloat16* out;
  int* status;
};

// Instruction descriptor, kind::f16, bf16 in, fp32 D; B MN-major (transposed)
__host__ __device__ constexpr uint32_t idesc_bf16_bmn(int M, int N) {
  return idesc_bf16(M, N) | (1u << 16);
}

// three-input maximum (one instruction on sm_100)
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Key k is visible from query q when 0 <= q - k < W; qk = q - (first key of
// the 32).  Keys past the sequence end never pass for a stored row q < T.
template <bool kMasked>
__device__ __forceinline__ void max32(const uint32_t (&v)[32], float (&mx)[8], int qk, int W) {
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    float x0 = __uint_as_float(v[e]), x1 = __uint_as_float(v[e + 1]);
    if (kMasked) {
      if ((unsigned)(qk - e) >= (unsigned)W) x0 = -INFINITY;
      if ((unsigned)(qk - e - 1) >= (unsigned)W) x1 = -INFINITY;
    }
    mx[(e >> 1) & 7] = fmax3f(mx[(e >> 1) & 7], x0, x1);
  }
}

// Row maximum of one S block (128 fp32 columns from TMEM), loads double
// buffered, eight independent max chains.
template <bool kMasked>
__device__ __forceinline__ float row_max(uint32_t s_addr, int qk, int W) {
  float mx[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) mx[e] = -INFINITY;
  uint32_t va[32], vb[32];
  tmem_ld32(s_addr, va);
  tmem_ld_wait_regs(va);
  tmem_ld32(s_addr + 32, vb);
  max32<kMasked>(va, mx, qk, W);
  tmem_ld_wait_regs(vb);
  tmem_ld32(s_addr + 64, va);
  max32<kMasked>(vb, mx, qk - 32, W);
  tmem_ld_wait_regs(va);
  tmem_ld32(s_addr + 96, vb);
  max32<kMasked>(va, mx, qk - 64, W);
  tmem_ld_wait_regs(vb);
  max32<kMasked>(vb, mx, qk - 96, W);
#pragma unroll
  for (int w = 4; w > 0; w >>= 1)
#pragma unroll
    for (int e = 0; e < w; ++e) mx[e] = fmaxf(mx[e], mx[e + w]);
  return mx[0];
}

// P = 2^(s * scale - base) of 32 keys as 16 packed bf16 pairs into TMEM; the
// scale and the row sums run as packed fp32x2 FMA / add (sm_100).
template <bool kMasked>
__device__ __forceinline__ void exp32(const uint32_t (&v)[32], float2 (&sum)[4], uint32_t p_addr,
                                      float2 sl2, float2 nbase, int qk, int W) {
  uint32_t pk[16];
#pragma unroll
  for (int e = 0; e < 32; e += 2) {
    const float2 x =
        __ffma2_rn(make_float2(__uint_as_float(v[e]), __uint_as_float(v[e + 1])), sl2, nbase);
    float p0 = exp2f(x.x), p1 = exp2f(x.y);
    if (kMasked) {
      if ((unsigned)(qk - e) >= (unsigned)W) p0 = 0.f;
      if ((unsigned)(qk - e - 1) >= (unsigned)W) p1 = 0.f;
    }
    sum[(e >> 1) & 3] = __fadd2_rn(sum[(e >> 1) & 3], make_float2(p0, p1));
    pk[e / 2] = pack2(p0, p1);
  }
  tmem_st16(p_addr, pk);
}

// P of one block into TMEM (64 columns); returns the row sum of P in fp32.
template <bool kMasked>
__device__ __forceinline__ float row_exp(uint32_t s_addr, uint32_t p_addr, float sl2, float base,
                                         int qk, int W) {
  float2 sum[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) sum[e] = make_float2(0.f, 0.f);
  const float2 s2 = make_float2(sl2, sl2), nb = make_float2(-base, -base);
  uint32_t va[32], vb[32];
  tmem_ld32(s_addr, va);
  tmem_ld_wait_regs(va);
  tmem_ld32(s_addr + 32, vb);
  exp32<kMasked>(va, sum, p_addr, s2, nb, qk, W);
  tmem_ld_wait_regs(vb);
  tmem_ld32(s_addr + 64, va);
  exp32<kMasked>(vb, sum, p_addr + 16, s2, nb, qk - 32, W);
  tmem_ld_wait_regs(va);
  tmem_ld32(s_addr + 96, vb);
  exp32<kMasked>(va, sum, p_addr + 32, s2, nb, qk - 64, W);
  tmem_ld_wait_regs(vb);
  exp32<kMasked>(vb, sum, p_addr + 48, s2, nb, qk - 96, W);
  const float2 t = __fadd2_rn(__fadd2_rn(sum[0], sum[1]), __fadd2_rn(sum[2], sum[3]));
  return t.x + t.y;
}

__global__ void __launch_bounds__(kAtThreads, 2)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, AtArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sKV = sQ + kAtTile;  // stage s: K at s*2*tile, V after it
  uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + kAtStages * 2 * kAtTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kAtStages;
  uint64_t* s_full = kv_empty + kAtStages;
  uint64_t* p_full = s_full + 1;
  uint64_t* o_done = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = a.T, d = a.H * kAtHd;
  const int q0 = qb * kAtBq;
  const bool windowed = a.window > 0 && a.window < T;
  const int W = windowed ? a.window : T + 1;
  int kstart = q0 - W + 1;
  if (kstart < 0) kstart = 0;
  kstart = (kstart / kAtBk) * kAtBk;
  const int kend = min(q0 + kAtBq, T);
  const int nblk = (kend - kstart + kAtBk - 1) / kAtBk;
  const int row0 = b * T;  // first row of this sequence in the (B*T, 3d) projection

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kAtStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    fence_barrier_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kAtCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) prefetch_tmap(&tmQKV);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    if (lane == 0) {  // ---------------- TMA producer
      bool ok = true;
      mbar_arrive_expect_tx(q_full, kAtTile);
      tma_load_2d(&tmQKV, q_full, sQ, h * kAtHd, row0 + q0);
      int s = 0;
      uint32_t ph = 0;
      long fills = 0;
      for (int i = 0; i < nblk && ok; ++i) {
        if (!mbar_wait(&kv_empty[s], ph ^ 1, a.status)) { ok = false; break; }
        uint8_t* st = sKV + s * 2 * kAtTile;
        const int k0 = kstart + i * kAtBk;
        mbar_arrive_expect_tx(&kv_full[s], 2 * kAtTile);
        tma_load_2d(&tmQKV, &kv_full[s], st, d + h * kAtHd, row0 + k0);
        tma_load_2d(&tmQKV, &kv_full[s], st + kAtTile, 2 * d + h * kAtHd, row0 + k0);
        ++fills;
        if (++s == kAtStages) { s = 0; ph ^= 1; }
      }
      // drain: no copy may still be writing shared memory when the CTA exits
      mbar_wait(q_full, 0, nullptr, 1u << 20);
      for (int j = 0; j < kAtStages; ++j) {
        const long n = fills / kAtStages + (j < fills % kAtStages ? 1 : 0);
        if (n > 0) mbar_wait(&kv_full[j], (uint32_t)((n - 1) & 1), nullptr, 1u << 20);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // ---------------- MMA issuer
      const uint32_t id_s = idesc_bf16(kAtBq, kAtBk);
      const uint32_t id_o = idesc_bf16_bmn(kAtBq, kAtHd);
      bool ok = mbar_wait(q_full, 0, a.status);
      int s = 0;
      uint32_t ph = 0;
      const uint32_t qa = smem_u32(sQ);
      for (int i = 0; i < nblk && ok; ++i) {
        if (!mbar_wait(&kv_full[s], ph, a.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t ka = smem_u32(sKV + s * 2 * kAtTile);
        const uint32_t va = ka + kAtTile;
#pragma unroll
        for (int k = 0; k < kAtHd / 16; ++k)  // S = Q K^T, both K-major
          umma_bf16(tmem + kAtS, sw128_desc(qa + k * 32), sw128_desc(ka + k * 32), id_s, k != 0);
        umma_commit(s_full);
        // P of this block is in TMEM once the softmax warps arrive
        if (!mbar_wait(p_full, (uint32_t)(i & 1), a.status)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < kAtBk / 16; ++k)  // O += P V: 16 keys = 8 P columns, 16 V rows
          umma_bf16_ts(tmem + kAtO, tmem + kAtP + k * 8, sw128_desc(va + k * 16 * 128), id_o,
                       (i | k) != 0);
        umma_commit(&kv_empty[s]);
        // s_full of the next block also covers this P V (a commit tracks every
        // earlier MMA of this thread); o_done only marks the last one
        if (i == nblk - 1) umma_commit(o_done);
        if (++s == kAtStages) { s = 0; ph ^= 1; }
      }
    }
  } else {  // ---------------- softmax / epilogue warps 0-3: row r = TMEM lane r
    const int r = warp * 32 + lane;
    const int qrow = q0 + r;
    const uint32_t lrow = tmem + ((uint32_t)(warp * 32) << 16);
    const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    for (int i = 0; i < nblk; ++i) {
      const int k0 = kstart + i * kAtBk;
      // every (query, key) pair of the block is inside the band: no mask (CTA-uniform)
      const bool inner = k0 + kAtBk - 1 <= q0 && q0 + kAtBq - 1 - k0 < W && k0 + kAtBk <= T;
      ok = ok && mbar_wait(s_full, (uint32_t)(i & 1), a.status);
      tc_fence_after();
      __syncwarp();  // the spin above may leave lanes apart; tcgen05.ld is warp-collective
      // pass 1: the row maximum of the raw scores (scale > 0 commutes with max)
      const int qk = qrow - k0;
      const float bm = inner ? row_max<false>(lrow + kAtS, qk, W) : row_max<true>(lrow + kAtS, qk, W);
      // the running base moves only when a score passes it by more than 8
      // (base 2): P stays below 256, exact enough in bf16, O and l are
      // rescaled far less often, and O / l is the same
      const float mcand = fmaxf(m, bm * sl2);
      const bool move = mcand > m + 8.f;  // true on the first visible key (m = -inf)
      const float mn = move ? mcand : m;
      const float base = mn == -INFINITY ? 0.f : mn;
      const float c = move ? exp2f(m - base) : 1.f;  // 0 when m was -inf
      // S of this block has landed, so the previous block's P V has finished
      // too (the commit behind s_full covers it): O is stable and P is free
      if (i > 0) {
        // tcgen05.ld/st are warp-collective: the whole warp rescales when any
        // of its rows' base moved (c is exactly 1 for the others)
        if (__any_sync(0xffffffffu, move)) {
#pragma unroll
          for (int cc = 0; cc < kAtHd; cc += 32) {
            uint32_t v[32];
            tmem_ld32(lrow + kAtO + cc, v);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) v[e] = __float_as_uint(__uint_as_float(v[e]) * c);
            tmem_st32(lrow + kAtO + cc, v);
          }
        }
      }
      m = mn;
      // pass 2: P = 2^(s * scale - m) as bf16 into TMEM, 32 keys (16 columns) at a time
      const float rs = inner ? row_exp<false>(lrow + kAtS, lrow + kAtP, sl2, base, qk, W)
                             : row_exp<true>(lrow + kAtS, lrow + kAtP, sl2, base, qk, W);
      l = l * c + rs;
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // epilogue: O / l of this row
    if (nblk > 0) {
      ok = ok && mbar_wait(o_done, 0, a.status);
      tc_fence_after();
    }
    __syncwarp();
    const float inv = l > 0.f ? 1.f / l : 0.f;
    uint32_t ov[kAtHd / 2];
#pragma unroll
    for (int cc = 0; cc < kAtHd; cc += 32) {
      uint32_t v[32];
      tmem_ld32(lrow + kAtO + cc, v);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; e += 2)
        ov[(cc + e) / 2] = pack2(__uint_as_float(v[e]) * inv, __uint_as_float(v[e + 1]) * inv);
    }
    if (qrow < T && ok) {
      uint4* dst = reinterpret_cast<uint4*>(a.out + ((size_t)row0 + qrow) * a.ldo + h * kAtHd);
#pragma unroll
      for (int j = 0; j < kAtHd / 8; ++j)
        dst[j] = make_uint4(ov[4 * j], ov[4 * j + 1], ov[4 * j + 2], ov[4 * j + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, kAtCols);
  }
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" int dh_window_attn_prefill_tc(const void* qkv, int ld, void* out, int ldo, int batch,
                                         int T, int H, int hd, int window, int* status,
                                         void* stream) {
  DH_REQUIRE(qkv && out, DH_ERR_ARG, "dh_window_attn_prefill_tc: null pointer");
  DH_REQUIRE(hd == kAtHd, DH_ERR_SHAPE, "dh_window_attn_prefill_tc: head_dim %d (64 only)", hd);
  DH_REQUIRE(ld % 8 == 0 && ldo % 8 == 0 && T > 0 && batch > 0 && ld >= 3 * H * hd,
             DH_ERR_SHAPE, "dh_window_attn_prefill_tc: bad sizes");
  DH_REQUIRE(aligned16(out), DH_ERR_ARG, "dh_window_attn_prefill_tc: out not 16-byte aligned");
  CUtensorMap tm;
  const uint64_t dims[2] = {(uint64_t)ld, (uint64_t)batch * T};
  const uint64_t strides[1] = {(uint64_t)ld * 2};
  const uint32_t box[2] = {kAtHd, 128};
  int rc = make_tmap_bf16(&tm, qkv, 2, dims, strides, box, true);
  if (rc) return rc;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmem);
    configured_dev = dev;
  }
  AtArgs a{T, H, window, ldo, reinterpret_cast<__nv_bfloat16*>(out), status};
  dim3 grid((T + kAtBq - 1) / kAtBq, H, batch);
  attn_tc_kernel<<<grid, kAtThreads, kAtSmem, reinterpret_cast<cudaStream_t>(stream)>>>(tm, a);
  return check_launch("attn_tc_kernel");
}

// Persistent tcgen05 GEMM for the prefill projections: C = A . W^T
// (A: M x K bf16 row-major activations, W: N x K bf16 row-major weights, as
// nn.Linear stores them), fp32 accumulation in tensor memory.
//
// Warp roles (224 threads, one CTA per SM):
//   warp 0      TMA producer: A and W tiles (128-byte swizzle) into a
//               STAGES-deep shared-memory ring, completion on mbarriers
//   warp 1      allocates 2 x BN TMEM columns; one thread issues
//               tcgen05.mma (M=128, N=BN, K=16) and commits stage releases
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (each warp owns its
//               32-lane TMEM quadrant), fused op, staged through shared
//               memory for coalesced global stores
//   warp 6      waits on the stage-full and accumulator-empty mbarriers and
//               hands each ready k-block to warp 1 through a named barrier:
//               an mbarrier wait in the issuing thread stalls the tensor
//               pipe (measured on B200: one satisfied try_wait per four
//               MMAs nearly triples their time), a named barrier does not
// The accumulator is double-buffered in TMEM so the epilogue of tile i
// overlaps the main loop of tile i+1.  Tiles are rasterised in bands of
// `band` column blocks so a band's weight slice stays resident in L2 while
// every row block streams past it.
#include "common.cuh"
#include "tma.cuh"

namespace dh {
namespace {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kEpiWarps = 4;
constexpr int kGemmThreads = 224;
constexpr int kHandoffBar = 1;  // named barrier between the MMA warp and the waiter warp

// Named barrier of the MMA and waiter warps that also ANDs a flag across
// them (all 64 threads execute it, once per k-block, in lockstep).
__device__ __forceinline__ bool handoff(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 64, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)ok), "n"(kHandoffBar)
      : "memory");
  return r != 0;
}
constexpr int kStgRow = 80;  // staging row pitch in bytes (64 B of data + pad)

enum { EPI_STORE = 0, EPI_RESIDUAL = 1, EPI_SWIGLU = 2 };

struct GemmArgs {
  int M, N, K;
  __nv_bfloat16* C;
  int ldc;
  const __nv_bfloat16* R;
  int ldr;
  int epi;
  int n_out;
  int band;
  int* err;
  uint32_t wait_limit;  // polls of each bounded wait before it reports a timeout
};

template <int BN>
struct Cfg {
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int SMEM = 1024 + STAGES * (A_BYTES + B_BYTES) + kEpiWarps * 32 * kStgRow +
                              8 * (2 * STAGES + 4) + 16;
};

__device__ __forceinline__ void tile_coords(int tile, int m_blocks, int n_blocks, int band,
                                            int& mb, int& nb) {
  const int per_band = band * m_blocks;
  const int bi = tile / per_band;
  const int r = tile - bi * per_band;
  const int rem = n_blocks - bi * band;
  const int w = rem < band ? rem : band;
  mb = r / w;
  nb = bi * band + (r - mb * w);
}

__device__ __forceinline__ float silu(float g) { return g / (1.0f + expf(-g)); }

// Residual chunk of the coalesced store pattern below (lane -> 16 B of row
// chunk>>2, part chunk&3), issued before the accumulator is read so the
// global-load latency overlaps the TMEM load and staging.
__device__ __forceinline__ void load_residual(uint4 (&res)[4], int lane, int row0, int col0,
                                              const GemmArgs& g) {
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int chunk = it * 32 + lane;
    const int row = row0 + (chunk >> 2), col = col0 + (chunk & 3) * 8;
    res[it] = make_uint4(0, 0, 0, 0);
    if (row < g.M && col + 8 <= g.n_out)
      res[it] = *reinterpret_cast<const uint4*>(g.R + (size_t)row * g.ldr + col);
  }
}

// write this lane's 32 values (its row) to staging, then store the warp's
// 32 x 32 block: 16-byte row-contiguous stores when the output rows are
// 16-byte aligned, otherwise one coalesced 64-byte row segment per store
__device__ __forceinline__ void stage_and_store(const float (&v)[32], uint8_t* stg, int lane,
                                                int row0, int col0, const GemmArgs& g,
                                                const uint4 (&res)[4]) {
  uint4* dst = reinterpret_cast<uint4*>(stg + lane * kStgRow);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float f[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) f[e] = v[j * 8 + e];
    dst[j] = pack8(f);
  }
  __syncwarp();
  const bool vec = (g.ldc % 8 == 0) && (g.epi != EPI_RESIDUAL || g.ldr % 8 == 0);
  if (vec) {
#pragma unroll
    for (int it = 0; it < 4; ++it) {
      const int chunk = it * 32 + lane;
      const int r = chunk >> 2, part = chunk & 3;
      const int row = row0 + r, col = col0 + part * 8;
      if (row >= g.M || col >= g.n_out) continue;
      uint4 val = *reinterpret_cast<const uint4*>(stg + r * kStgRow + part * 16);
      __nv_bfloat16* out = g.C + (size_t)row * g.ldc + col;
      if (col + 8 <= g.n_out) {
        if (g.epi == EPI_RESIDUAL) {
          float a[8], b[8];
          unpack8(val, a);
          unpack8(res[it], b);
#pragma unroll
          for (int e = 0; e < 8; ++e) a[e] += b[e];
          val = pack8(a);
        }
        *reinterpret_cast<uint4*>(out) = val;
      } else {
        const __nv_bfloat16* hv = reinterpret_cast<const __nv_bfloat16*>(&val);
        for (int e = 0; e < 8 && col + e < g.n_out; ++e) {
          float x = bf2f(hv[e]);
          if (g.epi == EPI_RESIDUAL) x += bf2f(g.R[(size_t)row * g.ldr + col + e]);
          out[e] = f2bf(x);
        }
      }
    }
  } else {
    const int col = col0 + lane;
    const bool col_ok = col < g.n_out;
    for (int r = 0; r < 32; ++r) {
      const int row = row0 + r;
      if (row >= g.M) break;
      if (!col_ok) continue;
      float x = bf2f(reinterpret_cast<const __nv_bfloat16*>(stg + r * kStgRow)[lane]);
      if (g.epi == EPI_RESIDUAL) x += bf2f(g.R[(size_t)row * g.ldr + col]);
      g.C[(size_t)row * g.ldc + col] = f2bf(x);
    }
  }
  __syncwarp();
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                GemmArgs g) {
  using C = Cfg<BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = sA + STAGES * C::A_BYTES;
  uint8_t* sStg = sB + STAGES * C::B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sStg + kEpiWarps * 32 * kStgRow);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m_blocks = (g.M + BM - 1) / BM, n_blocks = (g.N + BN - 1) / BN;
  const int num_tiles = m_blocks * n_blocks;
  const int kblocks = g.K / BK;
  const int band = g.band < n_blocks ? g.band : n_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], kEpiWarps);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&ta);
    prefetch_tmap(&tb);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long fills = 0;
      bool okk = true;
      for (int tile = blockIdx.x; tile < num_tiles && okk; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, m_blocks, n_blocks, band, mb, nb);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, g.err, g.wait_limit)) { okk = false; break; }
          mbar_arrive_expect_tx(&full[stage], C::A_BYTES + C::B_BYTES);
          tma_load_2d(&ta, &full[stage], sA + stage * C::A_BYTES, kb * BK, mb * BM);
          tma_load_2d(&tb, &full[stage], sB + stage * C::B_BYTES, kb * BK, nb * BN);
          ++fills;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // every issued fill must have landed before the CTA exits (only an
      // aborted run can leave one pending)
      for (int s = 0; s < STAGES; ++s) {
        const long n_s = fills / STAGES + (s < fills % STAGES ? 1 : 0);
        if (n_s > 0) mbar_wait(&full[s], (uint32_t)((n_s - 1) & 1), nullptr, 1u << 20);
      }
    }
  } else if (warp == 1) {  // ---------------- MMA issue (no mbarrier waits here)
    constexpr uint32_t idesc = idesc_bf16(BM, BN);
    int stage = 0, acc = 0;
    bool okk = true;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const uint32_t d_tmem = tmem_base + acc * BN;
      for (int kb = 0; kb < kblocks; ++kb) {
        okk = handoff(okk);  // the waiter saw this stage full (and, at kb 0, the accumulator free)
        tc_fence_after();
        if (okk && lane == 0) {
          const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
          const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            umma_bf16(d_tmem, sw128_desc(a0 + k * 32), sw128_desc(b0 + k * 32), idesc,
                      (kb | k) != 0);
          umma_commit(&empty[stage]);
          if (kb == kblocks - 1) umma_commit(&tfull[acc]);
        }
        __syncwarp();
        if (++stage == STAGES) stage = 0;
      }
      acc ^= 1;
    }
  } else if (warp == 6) {  // ---------------- waiter: mbarrier waits for the MMA warp
    int stage = 0, acc = 0;
    uint32_t phase = 0, acc_phase = 0;
    bool okk = true;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      for (int kb = 0; kb < kblocks; ++kb) {
        // after a failed (bounded) wait, skip every later wait but keep the
        // handoffs, so the two warps stay in lockstep and nothing blocks
        if (kb == 0) okk = okk && mbar_wait(&tempty[acc], acc_phase ^ 1, g.err, g.wait_limit);
        okk = okk && mbar_wait(&full[stage], phase, g.err, g.wait_limit);
        okk = handoff(okk);
        if (++stage == STAGES) { stage = 0; phase ^= 1; }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  } else {  // ---------------- epilogue warps 2..5
    const int q = warp & 3;
    uint8_t* stg = sStg + (warp - 2) * 32 * kStgRow;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      int mb, nb;
      tile_coords(tile, m_blocks, n_blocks, band, mb, nb);
      if (!mbar_wait(&tfull[acc], acc_phase, g.err, g.wait_limit)) break;
      tc_fence_after();
      const int row0 = mb * BM + q * 32;
      const uint32_t trow = tmem_base + ((uint32_t)(q * 32) << 16) + acc * BN;
      if (g.epi == EPI_SWIGLU) {
        const uint4 nores[4] = {};
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t gv[32], uv[32];
          tmem_ld32(trow + c, gv);
          tmem_ld32(trow + BN / 2 + c, uv);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = silu(__uint_as_float(gv[e])) * __uint_as_float(uv[e]);
          stage_and_store(v, stg, lane, row0, nb * (BN / 2) + c, g, nores);
        }
      } else {
        const bool resid = g.epi == EPI_RESIDUAL && (g.ldr % 8 == 0);
        uint4 res[4] = {};
        if (resid) load_residual(res, lane, row0, nb * BN, g);
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t rv[32];
          tmem_ld32(trow + c, rv);
          uint4 cur[4] = {res[0], res[1], res[2], res[3]};
          if (resid && c + 32 < BN) load_residual(res, lane, row0, nb * BN + c + 32, g);
          tmem_ld_wait();
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(rv[e]);
          stage_and_store(v, stg, lane, row0, nb * BN + c, g, cur);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::TMEM_COLS);
  }
}

template <int BN>
int launch_gemm(const void* A, int lda, const void* W, int ldw, GemmArgs g, cudaStream_t st) {
  CUtensorMap ta, tb;
  const uint64_t da[2] = {(uint64_t)g.K, (uint64_t)g.M}, sa[1] = {(uint64_t)lda * 2};
  const uint32_t ba[2] = {BK, BM};
  int rc = make_tmap_bf16(&ta, A, 2, da, sa, ba, true);
  if (rc) return rc;
  const uint64_t db[2] = {(uint64_t)g.K, (uint64_t)g.N}, sb[1] = {(uint64_t)ldw * 2};
  const uint32_t bb[2] = {BK, BN};
  rc = make_tmap_bf16(&tb, W, 2, db, sb, bb, true);
  if (rc) return rc;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(gemm_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         Cfg<BN>::SMEM);
    configured_dev = dev;
  }
  const int tiles = ((g.M + BM - 1) / BM) * ((g.N + BN - 1) / BN);
  int grid = sm_count();
  if (grid > tiles) grid = tiles;
  gemm_kernel<BN><<<grid, kGemmThreads, Cfg<BN>::SMEM, st>>>(ta, tb, g);
  return check_launch("gemm_kernel");
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" int dh_gemm_bf16(const void* A, int lda, const void* W, int ldw, void* C, int ldc,
                            const void* R, int ldr, int M, int N, int K, int epilogue,
                            int* status, void* stream) {
  DH_REQUIRE(A && W && C, DH_ERR_ARG, "dh_gemm_bf16: null pointer");
  DH_REQUIRE(M > 0 && N > 0 && K > 0 && K % BK == 0, DH_ERR_SHAPE,
             "dh_gemm_bf16: M=%d N=%d K=%d (K must be a multiple of 64)", M, N, K);
  DH_REQUIRE(lda % 8 == 0 && ldw % 8 == 0 && lda >= K && ldw >= K, DH_ERR_SHAPE,
             "dh_gemm_bf16: lda/ldw must be multiples of 8 and >= K");
  DH_REQUIRE(epilogue >= 0 && epilogue <= 2, DH_ERR_ARG, "dh_gemm_bf16: epilogue %d", epilogue);
  DH_REQUIRE(epilogue != EPI_RESIDUAL || R, DH_ERR_ARG, "dh_gemm_bf16: residual pointer missing");
  GemmArgs g{M, N, K, reinterpret_cast<__nv_bfloat16*>(C), ldc,
             reinterpret_cast<const __nv_bfloat16*>(R), ldr, epilogue, N, 16, status,
             wait_limit()};
  if (epilogue == EPI_SWIGLU) {
    DH_REQUIRE(N % 256 == 0, DH_ERR_SHAPE,
               "dh_gemm_bf16: SwiGLU needs N (= 2 ff) a multiple of 256, got %d", N);
    g.n_out = N / 2;
    DH_REQUIRE(ldc >= g.n_out, DH_ERR_SHAPE, "dh_gemm_bf16: ldc < ff");
    return launch_gemm<256>(A, lda, W, ldw, g, reinterpret_cast<cudaStream_t>(stream));
  }
  DH_REQUIRE(ldc >= N, DH_ERR_SHAPE, "dh_gemm_bf16: ldc < N");
  if (N <= 128)
    return launch_gemm<128>(A, lda, W, ldw, g, reinterpret_cast<cudaStream_t>(stream));
  return launch_gemm<256>(A, lda, W, ldw, g, reinterpret_cast<cudaStream_t>(stream));
}

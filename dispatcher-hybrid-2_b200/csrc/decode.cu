// Decode-step kernels: one lockstep position for batch <= 16 rows per launch
// (larger batches are split into chunks of 16 by the entry points).
//
// Every weight matrix is streamed from HBM exactly once per step.  The GEMVs
// and the FFN run on the tensor cores with the weights brought by bulk copies
// (gemv_bulk_kernel, ffn_bulk_kernel: the lockstep rows are the N side of
// mma.sync); the CUDA-core forms below them (a warp per pair of output rows,
// a transpose-reduction over the lockstep rows so that lane l ends up owning
// (row, batch) = (l / B, l % B)) take the shapes the tensor-core kernels do
// not, and the tree step for 1-2 rows.
#include <math.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace dh {
namespace {

constexpr int kGemvWarps = 8;
constexpr int kMaxRows = 16;  // rows of the batch handled per launch
constexpr float kNormEps = 1.1920928955078125e-07f;  // fp32 machine epsilon (torch RMSNorm, eps=None)

// Launch with programmatic stream serialization: the kernel may begin while
// its predecessor drains; every kernel here calls pdl_wait() before touching
// data that a predecessor writes.
template <typename Kern, typename... Args>
int launch_pdl(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess ? 0 : 1;
}

// After this, lane l holds the warp-wide sum of v[l % NV] (NV a power of two <= 32).
template <int NV>
__device__ __forceinline__ float transpose_reduce(float (&v)[NV]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = NV; n > 1; n >>= 1) {
    const int o = n >> 1;
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float r = v[0];
#pragma unroll
  for (int o = NV; o < 32; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

struct GemvIn {
  const void* x;                 // (batch, K): fp32 when x_f32, else bf16
  int x_f32;
  const __nv_bfloat16* norm_w;   // nullable: RMSNorm weight applied to x
  int K;
  int batch;
  int* status;                   // nullable: raised when a bounded wait gives up
};

// ---- epilogues: rows(u) names the two weight rows of work unit u;
//      store() receives, in each lane, the dot product of row `row` of unit u
//      with batch row b, and the partner row's value for the same b; bind()
//      runs once per thread at kernel start and reads what store() needs
//      from the device (the position t, stable within a step) off the
//      epilogue's critical path.
struct EpiMixerIn {  // W3 = [W_in; W1x; W1s], adjacent row pairs
  const __nv_bfloat16* w;
  int d, K, max_len;
  __nv_bfloat16 *v0, *a, *bh;
  const int64_t* t_buf;
  long long t;
  __device__ void bind() { t = *t_buf; }
  __device__ int units() const { return 3 * d / 2; }
  __device__ bool rows(int u, const __nv_bfloat16*& r0, const __nv_bfloat16*& r1) const {
    r0 = w + (size_t)(2 * u) * K;
    r1 = r0 + K;
    return true;
  }
  __device__ void store(int u, int b, int row, float v, float, bool) const {
    const int n = 2 * u + row, seg = n / d, c = n % d;
    if (seg == 0) v0[(size_t)b * d + c] = f2bf(v);
    else if (seg == 1) a[(size_t)b * d + c] = f2bf(v);
    else bh[((size_t)b * max_len + t) * d + c] = f2bf(v);
  }
};

struct EpiResidual {  // x[b, n] += v (and x_copy[b, n] = the new x when x_copy is set)
  const __nv_bfloat16* w;
  int N, K;
  float* x;
  float* x_copy;
  __device__ void bind() {}
  __device__ int units() const { return N / 2; }
  __device__ bool rows(int u, const __nv_bfloat16*& r0, const __nv_bfloat16*& r1) const {
    r0 = w + (size_t)(2 * u) * K;
    r1 = r0 + K;
    return true;
  }
  __device__ void store(int u, int b, int row, float v, float, bool) const {
    const size_t i = (size_t)b * N + 2 * u + row;
    const float nx = x[i] + v;
    x[i] = nx;
    if (x_copy) x_copy[i] = nx;
  }
};

struct EpiSwiglu {  // unit j = (gate row j, up row j) -> silu(g) * u
  const __nv_bfloat16 *wg, *wu;
  int ff, K;
  __nv_bfloat16* out;
  __device__ void bind() {}
  __device__ int units() const { return ff; }
  __device__ bool rows(int u, const __nv_bfloat16*& r0, const __nv_bfloat16*& r1) const {
    r0 = wg + (size_t)u * K;
    r1 = wu + (size_t)u * K;
    return true;
  }
  __device__ void store(int u, int b, int row, float v, float other, bool) const {
    if (row != 0) return;
    const float g = v, up = other;
    out[(size_t)b * ff + u] = f2bf(g / (1.0f + expf(-g)) * up);
  }
};

struct EpiQkvRope {  // [Wq; Wk; Wv], row pairs (2j, 2j+1) rotated for q and k
  const __nv_bfloat16* w;
  int d, K, hd, max_len;
  const float *cosT, *sinT;
  __nv_bfloat16 *q, *kc, *vc;
  const int64_t* t_buf;
  long long t;
  __device__ void bind() { t = *t_buf; }
  __device__ int units() const { return 3 * d / 2; }
  __device__ bool rows(int u, const __nv_bfloat16*& r0, const __nv_bfloat16*& r1) const {
    r0 = w + (size_t)(2 * u) * K;
    r1 = r0 + K;
    return true;
  }
  __device__ void store(int u, int b, int row, float v, float other, bool) const {
    const int n = 2 * u + row, seg = n / d, c = n % d;
    float out = v;
    if (seg < 2) {
      const int j = (c % hd) >> 1;
      const float cs = cosT[t * (hd / 2) + j], sn = sinT[t * (hd / 2) + j];
      const float x1 = row == 0 ? v : other, x2 = row == 0 ? other : v;
      out = row == 0 ? (x1 * cs - x2 * sn) : (x1 * sn + x2 * cs);
    }
    if (seg == 0) q[(size_t)b * d + c] = f2bf(out);
    else if (seg == 1) kc[((size_t)b * max_len + t) * d + c] = f2bf(out);
    else vc[((size_t)b * max_len + t) * d + c] = f2bf(out);
  }
};

struct EpiLogits {  // rows of E, odd vocab handled by a half-empty last unit
  const __nv_bfloat16* w;
  int V, K;
  __nv_bfloat16* out;
  __device__ void bind() {}
  __device__ int units() const { return (V + 1) / 2; }
  __device__ bool rows(int u, const __nv_bfloat16*& r0, const __nv_bfloat16*& r1) const {
    r0 = w + (size_t)(2 * u) * K;
    const bool has1 = 2 * u + 1 < V;
    r1 = has1 ? r0 + K : r0;
    return has1;
  }
  __device__ void store(int u, int b, int row, float v, float, bool has1) const {
    if (row == 1 && !has1) return;
    out[(size_t)b * V + 2 * u + row] = f2bf(v);
  }
};

template <int MAXB, class Epi>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(GemvIn in, Epi epi_in) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  Epi epi = epi_in;
  epi.bind();
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [batch][K]
  __shared__ float s_rstd[MAXB];
  pdl_trigger();
  const int K = in.K, batch = in.batch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nunits = epi.units();
  // each CTA owns a contiguous run of units, so its weight rows are contiguous
  const int upc = (nunits + gridDim.x - 1) / gridDim.x;
  const int u_begin = blockIdx.x * upc;
  const int u_end = min(nunits, u_begin + upc);

  // weights do not depend on the previous kernel: pull this warp's first row
  // pair into registers (and the rest of its rows into L2) while the producer
  // of x is still running
  // (only for one or two lockstep rows: from 4 rows on the registers cost
  // more occupancy than the head start gains)
  constexpr int kPre = MAXB <= 2 ? 4 : 0;  // 256-column iterations held in registers
  uint4 wpre[kPre > 0 ? 2 * kPre : 1];
  if (u_begin + warp < u_end) {
    const __nv_bfloat16 *r0, *r1;
    epi.rows(u_begin + warp, r0, r1);
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
      const int k = lane * 8 + i * 256;
      if (k < K) {
        wpre[2 * i] = ld_stream16(r0 + k);
        wpre[2 * i + 1] = ld_stream16(r1 + k);
      }
    }
    if (lane == 0) {
      for (int u = u_begin + warp + (kPre > 0 ? kGemvWarps : 0); u < u_end; u += kGemvWarps) {
        epi.rows(u, r0, r1);
        prefetch_l2(r0, (uint32_t)K * 2);
        prefetch_l2(r1, (uint32_t)K * 2);
      }
    }
  }
  pdl_wait();

  // one or two rows: the whole staging is one round trip per thread;
  // more rows: fewer registers keep two CTAs per SM
  if constexpr (MAXB <= 2) {
    if (in.x_f32) {
      // normalised input: every thread takes float4s of the rows (one L2 round
      // trip), squares are reduced per row in shared memory
      const float* x = static_cast<const float*>(in.x);
      const int k4 = K / 4, n4 = batch * k4;
      if (threadIdx.x < MAXB) s_rstd[threadIdx.x] = 0.f;
      __syncthreads();
      constexpr int NV = (MAXB * 1024) / (kGemvWarps * 32 * 4) > 0 ? (MAXB * 1024) / (kGemvWarps * 32 * 4) : 1;
      static_assert(NV <= 16, "row staging held in registers");
      float4 v[NV];
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int i = threadIdx.x + j * kGemvWarps * 32;
        float sq = 0.f;
        if (i < n4) {
          v[j] = reinterpret_cast<const float4*>(x)[i];
          sq = v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
        }
        if (in.norm_w) {
          if ((k4 & 31) == 0) {
            sq = warp_sum(sq);
            if (lane == 0 && i < n4) atomicAdd(&s_rstd[i / k4], sq);
          } else if (i < n4) {
            atomicAdd(&s_rstd[i / k4], sq);
          }
        }
      }
      __syncthreads();
#pragma unroll
      for (int j = 0; j < NV; ++j) {
        const int i = threadIdx.x + j * kGemvWarps * 32;
        if (i < n4) {
          const int b = i / k4, k = (i - b * k4) * 4;
          float4 q = v[j];
          if (in.norm_w) {
            const float r = rsqrtf(s_rstd[b] / (float)K + kNormEps);
            q.x = q.x * r * bf2f(in.norm_w[k]);
            q.y = q.y * r * bf2f(in.norm_w[k + 1]);
            q.z = q.z * r * bf2f(in.norm_w[k + 2]);
            q.w = q.w * r * bf2f(in.norm_w[k + 3]);
          }
          uint2 pk;
          pk.x = pack2(q.x, q.y);
          pk.y = pack2(q.z, q.w);
          *reinterpret_cast<uint2*>(xs + (size_t)b * K + k) = pk;
        }
      }
    } else {
      const uint4* x = static_cast<const uint4*>(in.x);
      const int n = batch * K / 8;
      for (int i0 = threadIdx.x; i0 < n; i0 += 8 * kGemvWarps * 32) {
        uint4 t8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + j * kGemvWarps * 32;
          if (i < n) t8[j] = x[i];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = i0 + j * kGemvWarps * 32;
          if (i < n) reinterpret_cast<uint4*>(xs)[i] = t8[j];
        }
      }
    }
  } else {
    if (in.x_f32) {
      // normalised input, row by row: one warp per row sums the squares, then
      // all threads scale and convert
      const float* x = static_cast<const float*>(in.x);
      if (in.norm_w) {
        for (int b = warp; b < batch; b += kGemvWarps) {
          const float4* xr = reinterpret_cast<const float4*>(x + (size_t)b * K);
          float ss = 0.f;
          for (int i = lane; i < K / 4; i += 32) {
            const float4 v = xr[i];
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
          }
          ss = warp_sum(ss);
          if (lane == 0) s_rstd[b] = rsqrtf(ss / (float)K + kNormEps);
        }
        __syncthreads();
      }
      const int k4 = K / 4;
      for (int i = threadIdx.x; i < batch * k4; i += blockDim.x) {
        const int b = i / k4, k = (i - b * k4) * 4;
        float4 v = reinterpret_cast<const float4*>(x + (size_t)b * K)[k / 4];
        if (in.norm_w) {
          const float r = s_rstd[b];
          v.x = v.x * r * bf2f(in.norm_w[k]);
          v.y = v.y * r * bf2f(in.norm_w[k + 1]);
          v.z = v.z * r * bf2f(in.norm_w[k + 2]);
          v.w = v.w * r * bf2f(in.norm_w[k + 3]);
        }
        uint2 pk;
        pk.x = pack2(v.x, v.y);
        pk.y = pack2(v.z, v.w);
        *reinterpret_cast<uint2*>(xs + (size_t)b * K + k) = pk;
      }
    } else {
      const uint4* x = static_cast<const uint4*>(in.x);
      for (int i = threadIdx.x; i < batch * K / 8; i += blockDim.x)
        reinterpret_cast<uint4*>(xs)[i] = x[i];
    }
  }
  __syncthreads();

  for (int u = u_begin + warp; u < u_end; u += kGemvWarps) {
    const __nv_bfloat16 *r0, *r1;
    const bool has1 = epi.rows(u, r0, r1);
    float acc[2 * MAXB];
#pragma unroll
    for (int i = 0; i < 2 * MAXB; ++i) acc[i] = 0.f;
    auto fma_chunk = [&](const uint4& wa, const uint4& wb, int k) {
      float fa[8], fb[8];
      unpack8(wa, fa);
      unpack8(wb, fb);
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        if (b < batch) {
          float fx[8];
          unpack8(*reinterpret_cast<const uint4*>(xs + (size_t)b * K + k), fx);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            acc[b] = fmaf(fa[j], fx[j], acc[b]);
            acc[MAXB + b] = fmaf(fb[j], fx[j], acc[MAXB + b]);
          }
        }
      }
    };
    const bool first = u == u_begin + warp;
#pragma unroll
    for (int i = 0; i < kPre; ++i) {
      const int k = lane * 8 + i * 256;
      if (k < K) {
        if (first) fma_chunk(wpre[2 * i], wpre[2 * i + 1], k);
        else fma_chunk(ld_stream16(r0 + k), ld_stream16(r1 + k), k);
      }
    }
#pragma unroll(MAXB <= 2 ? 4 : 2)
    for (int k = lane * 8 + kPre * 256; k < K; k += 256)
      fma_chunk(ld_stream16(r0 + k), ld_stream16(r1 + k), k);
    const float r = transpose_reduce<2 * MAXB>(acc);
    const float other = __shfl_xor_sync(0xffffffffu, r, MAXB);
    const int b = lane % MAXB, row = (lane / MAXB) & 1;
    if (lane < 2 * MAXB && b < batch) epi.store(u, b, row, r, other, has1);
  }
}

// ---------------------------------------------------------------- tensor-core GEMV
// The lockstep rows are the N side of mma.sync.m16n8k16 (bf16 in, fp32 out):
// one or two 8-column tiles for up to 8 or 16 rows, so a weight element
// costs 1/(8*16) of an instruction instead of 2*B FMAs.  A CTA takes 16-row
// tiles of the weight matrix (8 epilogue units: row pairs) in passes of 1024
// columns; its 8 consumer warps split a pass into 4 chunks of 32 columns
// each.  A producer warp streams the tiles with cp.async.bulk row copies into
// a ring of shared-memory slots (rows padded to 2112 bytes, so the fragment
// reads are bank-conflict free), completion on an mbarrier per slot.  One CTA
// per SM keeps up to six 33 KB slots in flight without holding weights in
// registers, and the producer starts before the predecessor kernel has
// finished (the weights do not depend on it).
//
// Fragments are plain 16-byte reads: lane (g, t4) reads columns
// [32c + 8 t4, +8) of tile rows g and g + 8.  The mma sums over the 16
// "logical" k of a k-step; which physical columns they are does not matter
// as long as the activation fragment uses the same ones, so k-step s of
// chunk c takes physical columns 32c + 8 t4 + 4s + {0,1} as logical k
// {2 t4, 2 t4 + 1} and 32c + 8 t4 + 4s + {2,3} as {2 t4 + 8, 2 t4 + 9} in
// both operands.  The activations sit in shared memory in natural column
// order, rows padded by 64 bytes.
constexpr int kTcWarps = 8;

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

constexpr int kBulkRowBytes = 2112;                // 1024 columns + 64 bytes of padding
constexpr int kBulkSlotBytes = 16 * kBulkRowBytes;  // one (tile, pass)
constexpr int kBulkMaxSlots = 6;
constexpr int kBulkThreads = (kTcWarps + 1) * 32;

struct BulkShared {
  uint64_t full[kBulkMaxSlots], empty[kBulkMaxSlots];
  int abort;
};

__host__ __device__ constexpr size_t bulk_xs_bytes(int nt, int K) { return (size_t)nt * 8 * (K + 32) * 2; }
__host__ __device__ constexpr size_t bulk_fixed_bytes(int nt, int K) {
  return bulk_xs_bytes(nt, K) + (size_t)kTcWarps * 16 * 16 * 4 + 16 * 17 * 4 + sizeof(BulkShared) + 16;
}

__device__ __forceinline__ void csync_bulk() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

template <int NT, class Epi>
__global__ void __launch_bounds__(kBulkThreads, 1)
    gemv_bulk_kernel(GemvIn in, Epi epi_in, int nslots, int wpt, int* status, uint32_t wait_limit) {
  extern __shared__ __align__(128) unsigned char bulk_smem[];
  Epi epi = epi_in;
  epi.bind();
  const int K = in.K, batch = in.batch, KP = K + 32;
  uint8_t* slots = bulk_smem;                                                 // [nslots][16][2112]
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(bulk_smem + (size_t)nslots * kBulkSlotBytes);
  float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + bulk_xs_bytes(NT, K));
  float* tile_out = red + kTcWarps * 16 * 16;                                // [16][17]
  BulkShared* sh = reinterpret_cast<BulkShared*>(tile_out + 16 * 17);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nunits = epi.units();
  const int ntiles = (nunits + 7) / 8;
  const int nchunks = K / 32;
  const int npass = (K + 1023) / 1024;
  const int nitems = (blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0) * npass;
  if (tid == 0) {
    for (int i = 0; i < nslots; ++i) {
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->empty[i], wpt ? 1 : kTcWarps);  // warp per tile: the slot's own warp
    }
    sh->abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kTcWarps) {  // ---------------- producer (one lane)
    if (lane != 0) return;
    int issued = 0;
    for (int item = 0; item < nitems; ++item) {
      const int slot = item % nslots;
      if (item >= nslots &&
          !mbar_wait(&sh->empty[slot], (uint32_t)(((item / nslots) - 1) & 1), status, wait_limit)) {
        sh->abort = 1;
        break;
      }
      if (*reinterpret_cast<volatile int*>(&sh->abort)) break;
      const int tile = blockIdx.x + (item / npass) * gridDim.x, pass = item % npass;
      const int cols = min(1024, K - pass * 1024);
      uint8_t* dst = slots + (size_t)slot * kBulkSlotBytes;
      mbar_arrive_expect_tx(&sh->full[slot], (uint32_t)(16 * cols * 2));
      for (int r = 0; r < 16; ++r) {
        const __nv_bfloat16 *a, *b;
        epi.rows(min(tile * 8 + (r >> 1), nunits - 1), a, b);
        const __nv_bfloat16* row = (r & 1) ? b : a;
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(dst + r * kBulkRowBytes)),
            "l"(row + pass * 1024), "r"((uint32_t)(cols * 2)), "r"(smem_u32(&sh->full[slot]))
            : "memory");
      }
      ++issued;
    }
    // no copy may still be in flight into this CTA's memory when it exits
    for (int sl = 0; sl < nslots; ++sl) {
      const int n_s = issued / nslots + (sl < issued % nslots ? 1 : 0);
      if (n_s > 0) mbar_wait(&sh->full[sl], (uint32_t)((n_s - 1) & 1), nullptr, 1u << 20);
    }
    return;
  }

  // ---------------- consumers (8 warps, named barrier 1)
  const int g = lane >> 2, t4 = lane & 3;
  pdl_wait();
  if (in.x_f32) {
    // warp w takes rows w and w + 8 whole: up to 1024 columns, 8 float4 per lane and row
    const float* x = static_cast<const float*>(in.x);
    const int k4 = K / 4;
    float4 v[NT][8];
    uint2 wn[8];
#pragma unroll
    for (int r = 0; r < NT; ++r) {
      const int b = warp + 8 * r;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = lane + 32 * j;
        v[r][j] = (b < batch && i < k4) ? reinterpret_cast<const float4*>(x + (size_t)b * K)[i]
                                        : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (in.norm_w) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = lane + 32 * j;
        wn[j] = i < k4 ? *reinterpret_cast<const uint2*>(in.norm_w + 4 * i) : make_uint2(0, 0);
      }
    }
#pragma unroll
    for (int r = 0; r < NT; ++r) {
      const int b = warp + 8 * r;
      float sc = 1.f;
      if (in.norm_w) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          ss += v[r][j].x * v[r][j].x + v[r][j].y * v[r][j].y + v[r][j].z * v[r][j].z + v[r][j].w * v[r][j].w;
        sc = rsqrtf(warp_sum(ss) / (float)K + kNormEps);
      }
      if (b < batch) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int i = lane + 32 * j;
          if (i < k4) {
            float4 q = v[r][j];
            if (in.norm_w) {
              const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wn[j].x));
              const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wn[j].y));
              q = make_float4(q.x * sc * w01.x, q.y * sc * w01.y, q.z * sc * w23.x, q.w * sc * w23.y);
            }
            uint2 pk;
            pk.x = pack2(q.x, q.y);
            pk.y = pack2(q.z, q.w);
            *reinterpret_cast<uint2*>(xs + (size_t)b * KP + 4 * i) = pk;
          }
        }
      }
    }
  } else {
    const int k8 = K / 8;
    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(in.x);
    for (int i = tid; i < batch * k8; i += kTcWarps * 32) {
      const int b = i / k8, k = (i - b * k8) * 8;
      asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(xs + (size_t)b * KP + k)),
                   "l"(x + (size_t)b * K + k)
                   : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
  }
  csync_bulk();

  if (wpt) {
    // warp per tile (one pass, many tiles per CTA): consumer warp w owns ring
    // slot w and takes items w, w + nslots, ... whole (every chunk of K, two
    // accumulator chains), so it never waits on its slot more than one fill
    // ahead; it releases the slot and stores its own results, with no
    // barrier and no cross-warp reduction per tile
    if (warp >= nslots) return;
    for (int item = warp; item < nitems; item += nslots) {
      const int slot = warp;
      const int tile = blockIdx.x + item * gridDim.x;
      bool ok = !*reinterpret_cast<volatile int*>(&sh->abort);
      if (ok && !mbar_wait(&sh->full[slot], (uint32_t)((item / nslots) & 1), status, wait_limit)) {
        sh->abort = 1;
        ok = false;
      }
      float ac[2][NT][4];
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) ac[q][nt][0] = ac[q][nt][1] = ac[q][nt][2] = ac[q][nt][3] = 0.f;
      if (ok) {
        const uint8_t* sb = slots + (size_t)slot * kBulkSlotBytes;
#pragma unroll 2
        for (int c = 0; c < nchunks; ++c) {
          const uint4 wa = *reinterpret_cast<const uint4*>(sb + g * kBulkRowBytes + c * 64 + t4 * 16);
          const uint4 wb = *reinterpret_cast<const uint4*>(sb + (g + 8) * kBulkRowBytes + c * 64 + t4 * 16);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)(nt * 8 + g) * KP + c * 32 + 8 * t4);
            mma_bf16_16816(ac[c & 1][nt], wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
            mma_bf16_16816(ac[c & 1][nt], wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[slot]);
      const bool live = ok && !*reinterpret_cast<volatile int*>(&sh->abort);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float v = ac[0][nt][e] + ac[1][nt][e];
          const float other = __shfl_xor_sync(0xffffffffu, v, 4);  // row g ^ 1, same column
          const int r = g + (e >> 1) * 8, b = nt * 8 + 2 * t4 + (e & 1);
          const int u = tile * 8 + (r >> 1);
          if (live && u < nunits && b < batch) {
            const __nv_bfloat16 *ra, *rb2;
            const bool has1 = epi.rows(u, ra, rb2);
            epi.store(u, b, r & 1, v, other, has1);
          }
        }
    }
    return;
  }
  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  for (int item = 0; item < nitems; ++item) {
    const int slot = item % nslots;
    const int tile = blockIdx.x + (item / npass) * gridDim.x, pass = item % npass;
    bool ok = !*reinterpret_cast<volatile int*>(&sh->abort);
    if (ok && !mbar_wait(&sh->full[slot], (uint32_t)((item / nslots) & 1), status, wait_limit)) {
      sh->abort = 1;
      ok = false;
    }
    if (ok) {
      const uint8_t* sb = slots + (size_t)slot * kBulkSlotBytes;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int cl = warp * 4 + i;  // chunk within the pass
        const int c = pass * 32 + cl;
        if (c < nchunks) {
          const uint4 wa = *reinterpret_cast<const uint4*>(sb + g * kBulkRowBytes + cl * 64 + t4 * 16);
          const uint4 wb = *reinterpret_cast<const uint4*>(sb + (g + 8) * kBulkRowBytes + cl * 64 + t4 * 16);
          uint4 xv[NT];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt)
            xv[nt] = *reinterpret_cast<const uint4*>(xs + (size_t)(nt * 8 + g) * KP + c * 32 + 8 * t4);
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            mma_bf16_16816(acc[nt], wa.x, wb.x, wa.y, wb.y, xv[nt].x, xv[nt].y);
            mma_bf16_16816(acc[nt], wa.z, wb.z, wa.w, wb.w, xv[nt].z, xv[nt].w);
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sh->empty[slot]);
    if (pass == npass - 1) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float* pr = red + (size_t)warp * 256;
        *reinterpret_cast<float2*>(pr + g * 16 + nt * 8 + 2 * t4) = make_float2(acc[nt][0], acc[nt][1]);
        *reinterpret_cast<float2*>(pr + (g + 8) * 16 + nt * 8 + 2 * t4) =
            make_float2(acc[nt][2], acc[nt][3]);
        acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
      }
      csync_bulk();
      {
        const int r = tid >> 4, col = tid & 15;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) s += red[w * 256 + r * 16 + col];
        tile_out[r * 17 + col] = s;
      }
      csync_bulk();
      {
        const int j = tid >> 5, row = (tid >> 4) & 1, b = tid & 15;
        const int u = tile * 8 + j;
        if (u < nunits && b < batch && !*reinterpret_cast<volatile int*>(&sh->abort)) {
          const __nv_bfloat16 *a, *bb;
          const bool has1 = epi.rows(u, a, bb);
          epi.store(u, b, row, tile_out[(2 * j + row) * 17 + b], tile_out[(2 * j + 1 - row) * 17 + b],
                    has1);
        }
      }
    }
  }
}

template <int NT, class Epi>
int launch_gemv_bulk(const GemvIn& in, const Epi& epi, int nunits, int* status, cudaStream_t st) {
  constexpr size_t kMaxSmem = 227 * 1024;
  const size_t fixed = bulk_fixed_bytes(NT, in.K);
  const int nslots = (int)std::min<size_t>(kBulkMaxSlots, (kMaxSmem - fixed) / kBulkSlotBytes);
  if (nslots < 2) return set_error(DH_ERR_SHAPE, "gemv: K=%d leaves no room for the weight ring", in.K);
  const size_t smem = fixed + (size_t)nslots * kBulkSlotBytes;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(gemv_bulk_kernel<NT, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kMaxSmem);
    configured_dev = dev;
  }
  const int ntiles = (nunits + 7) / 8;
  const int grid = std::min(ntiles, sm_count());
  // warp per tile when every CTA has 8 tiles or more of one pass (the logits)
  const int wpt = in.K <= 1024 && ntiles >= 8 * grid ? 1 : 0;
  return launch_pdl(gemv_bulk_kernel<NT, Epi>, dim3(grid), dim3(kBulkThreads), smem, st, in, epi, nslots,
                    wpt, status, wait_limit())
             ? set_error(DH_ERR_CUDA, "gemv_bulk_kernel launch: %s", cudaGetErrorString(cudaGetLastError()))
             : DH_OK;
}

template <int MAXB, class Epi>
int launch_gemv_b(const GemvIn& in, const Epi& epi, int nunits, cudaStream_t st) {
  const size_t smem = (size_t)MAXB * in.K * sizeof(__nv_bfloat16);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(gemv_kernel<MAXB, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kMaxRows * 2816 * 2 + 8192);
    configured_dev = dev;
  }
  int grid = (nunits + kGemvWarps - 1) / kGemvWarps;
  const int cap = sm_count() * 8;  // one resident wave of 256-thread CTAs
  if (grid > cap) grid = cap;
  return launch_pdl(gemv_kernel<MAXB, Epi>, dim3(grid), dim3(kGemvWarps * 32), smem, st, in, epi)
             ? set_error(DH_ERR_CUDA, "gemv_kernel launch: %s", cudaGetErrorString(cudaGetLastError()))
             : DH_OK;
}

template <class Epi>
int launch_gemv(GemvIn in, const Epi& epi, int nunits, cudaStream_t st) {
  if (in.K % 8 != 0 || in.K > 2816 * 2)
    return set_error(DH_ERR_SHAPE, "gemv: K=%d must be a multiple of 8 and <= 5632", in.K);
  if (in.x_f32 && in.K > 1024)
    return set_error(DH_ERR_SHAPE, "gemv: normalised input width %d exceeds 1024", in.K);
  if (in.batch <= 0 || in.batch > kMaxRows)
    return set_error(DH_ERR_SHAPE, "gemv: batch chunk %d outside [1, 16]", in.batch);
  if ((size_t)in.batch * in.K * 2 > (size_t)kMaxRows * 2816 * 2 + 8192)
    return set_error(DH_ERR_SHAPE, "gemv: batch*K too large for shared memory");
  if (in.K % 32 == 0 && aligned16(in.x)) {  // tensor cores, weights through the copy engine
    if (in.batch <= 8) return launch_gemv_bulk<1>(in, epi, nunits, in.status, st);
    return launch_gemv_bulk<2>(in, epi, nunits, in.status, st);
  }
  if (in.batch == 1) return launch_gemv_b<1>(in, epi, nunits, st);
  if (in.batch == 2) return launch_gemv_b<2>(in, epi, nunits, st);
  if (in.batch <= 4) return launch_gemv_b<4>(in, epi, nunits, st);
  if (in.batch <= 8) return launch_gemv_b<8>(in, epi, nunits, st);
  return launch_gemv_b<16>(in, epi, nunits, st);
}

// ---------------------------------------------------------------- tree step
struct TreeStepParams {
  const __nv_bfloat16 *a, *bh, *wi, *wf, *wr;
  const float *bi, *bf, *br;
  const int64_t* t_buf;
  float *ig, *fg;
  __nv_bfloat16* rg;
  const __nv_bfloat16* v0;
  __nv_bfloat16* ring;
  __nv_bfloat16* y;
  int* counters;
  const int* doc;  // nullable: document id per (row, position), (batch, max_len)
  int batch, max_len, L, H, hd, gh, S;
};

// grid (L, H): block (level l, head h) forms the three gate readouts of head h
// at level l for every row, then the last of the L blocks of head h to finish
// runs the level recurrence of head h (no block ever waits on another).
constexpr int kTreeGroups = 8;  // 8-channel groups per head (hd <= 64)

template <int MAXB>
__global__ void __launch_bounds__(128) tree_step_kernel(TreeStepParams p) {
  constexpr int LMAX = 16;
  const int l = blockIdx.x, h = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int L = p.L, H = p.H, gh = p.gh, d = H * p.hd;
  pdl_trigger();
  // t_buf is only advanced by the last kernel of a step, and the history rows
  // at positions < t were written by earlier steps: both are safe to read
  // before waiting on the producer of A / v0.
  const long long t = *p.t_buf;
  const long long src = t - (1ll << l);
  const bool ok = src >= 0;
  const long long srcc = ok ? src : 0;
  const size_t wrow = ((size_t)l * H + h) * gh;
  if (tid == 0) {
    prefetch_l2(p.wi + wrow, gh * 2);
    prefetch_l2(p.wf + wrow, gh * 2);
    prefetch_l2(p.wr + wrow, gh * 2);
  } else if (ok && tid <= p.batch) {
    const int b = tid - 1;
    prefetch_l2(p.bh + ((size_t)b * p.max_len + srcc) * gh, gh * 2);
    const long long slot = ((2ll << l) - 2) + (srcc & ((2ll << l) - 1));
    prefetch_l2(p.ring + ((size_t)b * p.S + slot) * d + h * p.hd, p.hd * 2);
  }
  pdl_wait();

  // per-row level mask: the source position exists and, with document
  // tracking, lies in the same document (the parallel forward's doc-reset
  // mask, modeling_dispatcher.py:311-323)
  __shared__ bool s_ok[MAXB];
  if (tid < MAXB) {
    bool okb = ok && tid < p.batch;
    if (okb && p.doc)
      okb = p.doc[(size_t)tid * p.max_len + srcc] == p.doc[(size_t)tid * p.max_len + t];
    s_ok[tid] = okb;
  }
  __syncthreads();
  float acc[MAXB][3];
#pragma unroll
  for (int b = 0; b < MAXB; ++b) acc[b][0] = acc[b][1] = acc[b][2] = 0.f;
  for (int k = tid * 8; k < gh; k += 128 * 8) {
    float fi[8], ff[8], fr[8];
    unpack8(ld_stream16(p.wi + wrow + k), fi);
    unpack8(ld_stream16(p.wf + wrow + k), ff);
    unpack8(ld_stream16(p.wr + wrow + k), fr);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < p.batch) {
        float fa[8], fs[8];
        unpack8(*reinterpret_cast<const uint4*>(p.a + (size_t)b * gh + k), fa);
        if (s_ok[b]) {
          unpack8(*reinterpret_cast<const uint4*>(p.bh + ((size_t)b * p.max_len + srcc) * gh + k),
                  fs);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) fs[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float hv = fmaxf(fa[j] + fs[j], 0.f);
          hv *= hv;  // relu squared
          acc[b][0] = fmaf(fi[j], hv, acc[b][0]);
          acc[b][1] = fmaf(ff[j], hv, acc[b][1]);
          acc[b][2] = fmaf(fr[j], hv, acc[b][2]);
        }
      }
    }
  }
  __shared__ float red[4][MAXB * 3];
#pragma unroll
  for (int b = 0; b < MAXB; ++b) {
#pragma unroll
    for (int g = 0; g < 3; ++g) {
      const float v = warp_sum(acc[b][g]);
      if (lane == 0) red[warp][b * 3 + g] = v;
    }
  }
  __syncthreads();
  if (tid < p.batch) {
    const int b = tid;
    float pre[3];
#pragma unroll
    for (int g = 0; g < 3; ++g) pre[g] = red[0][b * 3 + g] + red[1][b * 3 + g] + red[2][b * 3 + g] + red[3][b * 3 + g];
    const int lh = l * H + h;
    const float okf = s_ok[b] ? 1.f : 0.f;
    const float ig = sigmoidf_(pre[0] + p.bi[lh]) * okf;
    const float fg = sigmoidf_(pre[1] + p.bf[lh]) * okf + (1.f - okf);
    const float rg = sigmoidf_(pre[2] + p.br[lh]);
    p.ig[((size_t)b * L + l) * H + h] = ig;
    p.fg[((size_t)b * L + l) * H + h] = fg;
    p.rg[(((size_t)b * p.max_len + t) * L + l) * H + h] = f2bf(rg);
    __threadfence();
  }
  __syncthreads();
  __shared__ int s_last;
  if (tid == 0) s_last = (atomicAdd(&p.counters[h], 1) == L - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // level recurrence for head h (fused_step.py:62-88 semantics, fp32 state).
  // First every level's inputs are fetched in parallel (one round trip: the
  // ring slots read, positions t - 2^l, never coincide with the slots
  // written, position t), then a short serial chain runs from shared memory.
  __shared__ float s_f[MAXB][LMAX], s_c[MAXB][LMAX];
  __shared__ uint4 s_v[MAXB][LMAX][kTreeGroups];
  const int groups = p.hd / 8;
#pragma unroll 4
  for (int item = tid; item < p.batch * L * groups; item += blockDim.x) {
    const int b = item / (L * groups), rem = item - b * (L * groups);
    const int lv = rem / groups, g = rem - lv * groups;
    const long long s = t - (1ll << lv);
    uint4 vs = make_uint4(0, 0, 0, 0);
    if (s >= 0) {
      const long long slot = ((2ll << lv) - 2) + (s & ((2ll << lv) - 1));
      vs = *reinterpret_cast<const uint4*>(p.ring + ((size_t)b * p.S + slot) * d + h * p.hd +
                                           g * 8);
    }
    s_v[b][lv][g] = vs;
    if (g == 0) {
      s_f[b][lv] = __ldcg(p.fg + ((size_t)b * L + lv) * H + h);
      s_c[b][lv] = s >= 0 ? __ldcg(p.ig + ((size_t)b * L + lv) * H + h) *
                                bf2f(p.rg[(((size_t)b * p.max_len + s) * L + lv) * H + h])
                          : 0.f;
    }
  }
  __syncthreads();
  for (int idx = tid; idx < p.batch * groups; idx += blockDim.x) {
    const int b = idx / groups, g = idx - b * groups;
    const int c0 = h * p.hd + g * 8;
    __nv_bfloat16* ringb = p.ring + (size_t)b * p.S * d;
    float V[8];
    const uint4 v0 = *reinterpret_cast<const uint4*>(p.v0 + (size_t)b * d + c0);
    unpack8(v0, V);
    *reinterpret_cast<uint4*>(ringb + (size_t)(t & 1) * d + c0) = v0;  // ring 0 at t
    for (int lv = 0; lv < L; ++lv) {
      float vs[8];
      unpack8(s_v[b][lv][g], vs);
      const float f = s_f[b][lv], c = s_c[b][lv];
#pragma unroll
      for (int j = 0; j < 8; ++j) V[j] = f * V[j] + c * vs[j];
      if (lv + 1 < L) {
        const long long slot = ((2ll << (lv + 1)) - 2) + (t & ((2ll << (lv + 1)) - 1));
        *reinterpret_cast<uint4*>(ringb + (size_t)slot * d + c0) = pack8(V);
      }
    }
    *reinterpret_cast<uint4*>(p.y + (size_t)b * d + c0) = pack8(V);
  }
  if (tid == 0) p.counters[h] = 0;
}

// ---------------------------------------------------------------- tree step, 3..16 rows
// Gate readouts on the tensor cores.  For one level l the readouts of every
// head and gate form one GEMM: D (NP x B) = W_l (NP x gh) . hv_l (gh x B),
// with W_l the packed rows g*H + h (NP = 3H padded to 16) and hv_l[k, b] =
// relu(A[b, k] + B_hist[b, t - 2^l, k])^2 in bf16 (zero history where the
// source position is missing or in another document).  hv_l is formed once
// per level and column, for all heads.  Grid (L, gh / 256): each CTA adds
// its 256-column share into the fp32 pre-activations with atomics; the
// recurrence kernel that follows reads them and leaves zeros behind.
struct TreeGatesTcParams {
  const __nv_bfloat16 *a, *bh, *w;
  const int64_t* t_buf;
  const int* doc;  // nullable
  float* pre;      // (batch, L, NP) fp32, zero on entry
  const __nv_bfloat16* ring;  // V_ring (batch, S, d): the recurrence's history, prefetched here
  int batch, max_len, L, NP, gh, S, d;
};

template <int MT>
__global__ void __launch_bounds__(256) tree_gates_tc_kernel(TreeGatesTcParams p) {
  // the 8 warps' partial tiles meet in one tile through shared-memory adds:
  // 3 KB of static shared memory, small enough for the CTA to be resident
  // beside the W3 GEMV it follows and load its gate weights before that ends
  __shared__ float red[MT * 16][16];
  __shared__ bool s_ok[16];
  pdl_trigger();
  const int l = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int i = tid; i < MT * 16 * 16; i += blockDim.x) (&red[0][0])[i] = 0.f;
  const int g = lane >> 2, t4 = lane & 3;
  const int gh = p.gh, NP = p.NP;
  const long long t = *p.t_buf;  // advanced only by the last kernel of a step
  const long long src = t - (1ll << l);
  // this warp's 32 columns (warps past gh contribute zeros)
  const bool live = (blockIdx.y * kTcWarps + warp) * 32 < gh;
  const int k0 = live ? (blockIdx.y * kTcWarps + warp) * 32 + 8 * t4 : 0;
  // gate weights: independent of the earlier kernels of the step
  uint4 wa[MT], wb[MT];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    const size_t r = (size_t)l * NP + mt * 16 + g;
    wa[mt] = live ? ld_stream16(p.w + r * gh + k0) : make_uint4(0, 0, 0, 0);
    wb[mt] = live ? ld_stream16(p.w + (r + 8) * gh + k0) : make_uint4(0, 0, 0, 0);
  }
  // rows written by earlier steps that this level needs, into L2 while the
  // predecessor runs: each lockstep row's B_hist row at t - 2^l (read below)
  // and its ring slot of level l at t - 2^l (read by the recurrence kernel)
  if (blockIdx.y == 0 && src >= 0 && tid < 2 * p.batch) {
    const int b = tid >> 1;
    if (tid & 1) {
      const long long slot = ((2ll << l) - 2) + (src & ((2ll << l) - 1));
      prefetch_l2(p.ring + ((size_t)b * p.S + slot) * p.d, (uint32_t)p.d * 2);
    } else {
      prefetch_l2(p.bh + ((size_t)b * p.max_len + src) * gh, (uint32_t)gh * 2);
    }
  }
  pdl_wait();
  if (tid < 16) {
    bool ok = src >= 0 && tid < p.batch;
    if (ok && p.doc) ok = p.doc[(size_t)tid * p.max_len + src] == p.doc[(size_t)tid * p.max_len + t];
    s_ok[tid] = ok;
  }
  __syncthreads();
  // hv fragments of lockstep rows n = g and g + 8 for this lane's 8 columns
  uint32_t hv[2][4];
  const __nv_bfloat162 z2 = __floats2bfloat162_rn(0.f, 0.f);
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int n = nt * 8 + g;
    uint4 av = make_uint4(0, 0, 0, 0), bv = make_uint4(0, 0, 0, 0);
    if (live && n < p.batch) {
      av = *reinterpret_cast<const uint4*>(p.a + (size_t)n * gh + k0);
      if (s_ok[n]) bv = *reinterpret_cast<const uint4*>(p.bh + ((size_t)n * p.max_len + src) * gh + k0);
    }
    const uint32_t* ap = &av.x;
    const uint32_t* bp = &bv.x;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __hmax2(__hadd2(*reinterpret_cast<const __nv_bfloat162*>(ap + i),
                                         *reinterpret_cast<const __nv_bfloat162*>(bp + i)),
                                 z2);
      h = __hmul2(h, h);  // relu squared, rounded to bf16
      hv[nt][i] = n < p.batch ? *reinterpret_cast<uint32_t*>(&h) : 0u;
    }
  }
  float acc[MT][2][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      acc[mt][nt][0] = acc[mt][nt][1] = acc[mt][nt][2] = acc[mt][nt][3] = 0.f;
      mma_bf16_16816(acc[mt][nt], wa[mt].x, wb[mt].x, wa[mt].y, wb[mt].y, hv[nt][0], hv[nt][1]);
      mma_bf16_16816(acc[mt][nt], wa[mt].z, wb[mt].z, wa[mt].w, wb[mt].w, hv[nt][2], hv[nt][3]);
    }
#pragma unroll
  for (int mt = 0; mt < MT; ++mt)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
      atomicAdd(&red[mt * 16 + g][nt * 8 + 2 * t4], acc[mt][nt][0]);
      atomicAdd(&red[mt * 16 + g][nt * 8 + 2 * t4 + 1], acc[mt][nt][1]);
      atomicAdd(&red[mt * 16 + g + 8][nt * 8 + 2 * t4], acc[mt][nt][2]);
      atomicAdd(&red[mt * 16 + g + 8][nt * 8 + 2 * t4 + 1], acc[mt][nt][3]);
    }
  __syncthreads();
  for (int i = tid; i < MT * 16 * 16; i += blockDim.x) {
    const int m = i >> 4, n = i & 15;
    if (n < p.batch) atomicAdd(p.pre + ((size_t)n * p.L + l) * NP + m, red[m][n]);
  }
}

// Level recurrence of one (head, row): one thread per channel, every level's
// history value fetched up front (ring slots of earlier positions, written by
// earlier steps), then the short serial chain (fused_step.py:62-88 semantics,
// fp32 state, each level's value stored into its ring slot at t).

struct TreeRecurParams {
  float* pre;  // (batch, L, NP): read and cleared
  const float *bi, *bf, *br;
  const int64_t* t_buf;
  const int* doc;  // nullable
  __nv_bfloat16* rg;
  const __nv_bfloat16* v0;
  __nv_bfloat16* ring;
  __nv_bfloat16* y;
  int batch, max_len, L, H, hd, NP, S;
};

template <int RPB>
__global__ void __launch_bounds__(64 * RPB) tree_recur_kernel(TreeRecurParams p) {
  constexpr int LMAX = 16;
  __shared__ float s_f_all[RPB][LMAX], s_c_all[RPB][LMAX];
  pdl_trigger();
  const int h = blockIdx.x, b = blockIdx.y * blockDim.y + threadIdx.y, c = threadIdx.x;
  float* s_f = s_f_all[threadIdx.y];
  float* s_c = s_c_all[threadIdx.y];  // blockDim.y == p.batch: every thread has a row
  const int L = p.L, H = p.H, hd = p.hd, d = H * hd;
  const int t = (int)*p.t_buf;  // < max_len: positions and slots fit 32 bits
  __nv_bfloat16* ringb = p.ring + (size_t)b * p.S * d + h * hd + c;
  float vs[LMAX];
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
    const int s = t - (1 << l);
    vs[l] = 0.f;
    if (l < L && s >= 0 && c < hd) vs[l] = bf2f(ringb[(size_t)(((2 << l) - 2) + (s & ((2 << l) - 1))) * d]);
  }
  float rg_src = 0.f;
  if (c < L) {
    const int s = t - (1 << c);
    if (s >= 0) rg_src = bf2f(p.rg[(((size_t)b * p.max_len + s) * L + c) * H + h]);
  }
  pdl_wait();
  const __nv_bfloat16 v0 = c < hd ? p.v0[(size_t)b * d + h * hd + c] : __float2bfloat16(0.f);
  if (c < L) {
    const int l = c;
    const int s = t - (1 << l);
    bool ok = s >= 0;
    if (ok && p.doc) ok = p.doc[(size_t)b * p.max_len + s] == p.doc[(size_t)b * p.max_len + t];
    float* pr = p.pre + ((size_t)b * L + l) * p.NP;
    const float pi = pr[h], pf = pr[H + h], prr = pr[2 * H + h];
    pr[h] = 0.f;
    pr[H + h] = 0.f;
    pr[2 * H + h] = 0.f;
    const float okf = ok ? 1.f : 0.f;
    const int lh = l * H + h;
    const float ig = sigmoidf_(pi + p.bi[lh]) * okf;
    const float fg = sigmoidf_(pf + p.bf[lh]) * okf + (1.f - okf);
    const float rgt = sigmoidf_(prr + p.br[lh]);
    p.rg[(((size_t)b * p.max_len + t) * L + l) * H + h] = f2bf(rgt);
    s_f[l] = fg;
    s_c[l] = ig * rg_src;
  }
  __syncthreads();
  if (c >= hd) return;
  float V = bf2f(v0);
  ringb[(size_t)(t & 1) * d] = v0;  // ring 0 at t
#pragma unroll
  for (int l = 0; l < LMAX; ++l) {
    if (l < L) {
      V = s_f[l] * V + s_c[l] * vs[l];
      if (l + 1 < L) ringb[(size_t)(((2 << (l + 1)) - 2) + (t & ((2 << (l + 1)) - 1))) * d] = f2bf(V);
    }
  }
  p.y[(size_t)b * d + h * hd + c] = f2bf(V);
}

// RPB rows per block: every row of a head in one block for 1-4 lockstep
// rows (measured faster there), one block per (head, row) above
constexpr int kRecurRows = 16;

template <int RPB>
int launch_tree_recur(const TreeRecurParams& rp, int H, int nb, cudaStream_t st) {
  return RPB == 1 ? launch_pdl(tree_recur_kernel<1>, dim3(H, nb), dim3(64), 0, st, rp)
                  : launch_pdl(tree_recur_kernel<RPB>, dim3(H, 1), dim3(64, nb), 0, st, rp);
}

// ---------------------------------------------------------------- W3 GEMV with the gate readouts
// The tree block's input side and its gate readouts in one launch (1-8
// lockstep rows).  The W3 GEMV of the bulk-copy kernel above (v0, A, B_hist
// rows), and for every tile that produces 16 columns k of A, one more ring
// item: rows k of the transposed gate weights, all (level, gate, head)
// readouts at once (one bulk copy of 16 x L*NP bf16).  The readouts are sums
// over k, so the tile adds its share into the fp32 pre-activations:
//   pre[b, l*NP + g*H + h] += sum_k W_g[l, h, k] * relu(A[b, k] + m B_hist[b, t - 2^l, k])^2
// with A rounded to bf16 as stored, m the level mask (source position exists
// and, with document tracking, lies in the same document), fp32 arithmetic
// as in the (level, head) tree kernel.  The level recurrence then runs in
// tree_recur_kernel, which reads and clears pre.  The gate weights are read
// once per step in total; no hidden vector of the gates exists in HBM.
struct MixerGatesParams {
  const float* x;
  const __nv_bfloat16 *norm_w, *w3;
  __nv_bfloat16 *v0, *a, *bh;
  const int64_t* t_buf;
  const __nv_bfloat16* wgT;  // (d, L*NP): row k, column l*NP + g*H + h = W_g[l, h, k]
  float* pre;                // (batch, L*NP)
  const int* doc;            // nullable
  int d, batch, max_len, L, NP, H3;
};

constexpr int kGateMaxL = 16;

template <int NT>
__global__ void __launch_bounds__(kBulkThreads, 1)
    mixer_gates_kernel(MixerGatesParams p, int nslots, int* status, uint32_t wait_limit) {
  extern __shared__ __align__(128) unsigned char mg_smem[];
  const int d = p.d, K = d, KP = K + 32, batch = p.batch, LNP = p.L * p.NP;
  uint8_t* slots = mg_smem;                                                  // [nslots][16][2112]
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(mg_smem + (size_t)nslots * kBulkSlotBytes);
  float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + bulk_xs_bytes(NT, K));
  float* tile_out = red + kTcWarps * 16 * 16;  // [16][17]
  float* hv = tile_out + 16 * 17;              // [8 NT][kGateMaxL][16]
  BulkShared* sh = reinterpret_cast<BulkShared*>(hv + NT * 8 * kGateMaxL * 16);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nunits = 3 * d / 2, ntiles = 3 * d / 16, nchunks = K / 32;
  const int a_lo = d / 16, a_hi = 2 * d / 16;  // tiles whose rows are A
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int t = (int)*p.t_buf;  // advanced only by the last kernel of a step
  if (tid == 0) {
    for (int i = 0; i < nslots; ++i) {
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->empty[i], kTcWarps);
    }
    sh->abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kTcWarps) {  // ---------------- producer (one lane)
    if (lane != 0) return;
    int it = 0;
    for (int tl = 0; tl < my_tiles && !*reinterpret_cast<volatile int*>(&sh->abort); ++tl) {
      const int tile = blockIdx.x + tl * gridDim.x;
      const int nit = (tile >= a_lo && tile < a_hi) ? 2 : 1;
      for (int q = 0; q < nit; ++q, ++it) {
        const int slot = it % nslots;
        if (it >= nslots &&
            !mbar_wait(&sh->empty[slot], (uint32_t)(((it / nslots) - 1) & 1), status, wait_limit)) {
          sh->abort = 1;
          break;
        }
        uint8_t* dst = slots + (size_t)slot * kBulkSlotBytes;
        if (q == 0) {  // 16 rows of W3
          mbar_arrive_expect_tx(&sh->full[slot], (uint32_t)(16 * K * 2));
          for (int r = 0; r < 16; ++r)
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_u32(dst + r * kBulkRowBytes)),
                "l"(p.w3 + (size_t)(tile * 16 + r) * K), "r"((uint32_t)(K * 2)),
                "r"(smem_u32(&sh->full[slot]))
                : "memory");
        } else {  // rows k0..k0+15 of the transposed gate weights, contiguous
          const uint32_t bytes = (uint32_t)(16 * LNP * 2);
          mbar_arrive_expect_tx(&sh->full[slot], bytes);
          asm volatile(
              "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                  smem_u32(dst)),
              "l"(p.wgT + (size_t)(tile * 16 - d) * LNP), "r"(bytes), "r"(smem_u32(&sh->full[slot]))
              : "memory");
        }
      }
    }
    for (int sl = 0; sl < nslots; ++sl) {  // nothing in flight into this CTA when it exits
      const int n_s = it / nslots + (sl < it % nslots ? 1 : 0);
      if (n_s > 0) mbar_wait(&sh->full[sl], (uint32_t)((n_s - 1) & 1), nullptr, 1u << 20);
    }
    return;
  }

  // ---------------- consumers (8 warps, named barrier 1)
  const int g = lane >> 2, t4 = lane & 3;
  pdl_wait();
  {  // RMSNorm(x) rows as bf16, warp per row (up to 1024 columns)
    const int k4 = K / 4;
    for (int rb = warp; rb < batch; rb += kTcWarps) {
      const float* xr = p.x + (size_t)rb * K;
      float4 v[8];
      uint2 wn[8];
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < k4 ? reinterpret_cast<const float4*>(xr)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        wn[j] = i < k4 ? *reinterpret_cast<const uint2*>(p.norm_w + 4 * i) : make_uint2(0, 0);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
      const float sc = rsqrtf(warp_sum(ss) / (float)K + kNormEps);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = lane + 32 * j;
        if (i < k4) {
          const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wn[j].x));
          const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wn[j].y));
          uint2 pk;
          pk.x = pack2(v[j].x * sc * w01.x, v[j].y * sc * w01.y);
          pk.y = pack2(v[j].z * sc * w23.x, v[j].w * sc * w23.y);
          *reinterpret_cast<uint2*>(xs + (size_t)rb * KP + 4 * i) = pk;
        }
      }
    }
  }
  csync_bulk();

  int it = 0;
  for (int tl = 0; tl < my_tiles; ++tl) {
    const int tile = blockIdx.x + tl * gridDim.x;
    {  // ---- the W3 tile
      const int slot = it % nslots;
      bool ok = !*reinterpret_cast<volatile int*>(&sh->abort);
      if (ok && !mbar_wait(&sh->full[slot], (uint32_t)((it / nslots) & 1), status, wait_limit)) {
        sh->abort = 1;
        ok = false;
      }
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
      if (ok) {
        const uint8_t* sb = slots + (size_t)slot * kBulkSlotBytes;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = warp * 4 + i;
          if (c < nchunks) {
            const uint4 wa = *reinterpret_cast<const uint4*>(sb + g * kBulkRowBytes + c * 64 + t4 * 16);
            const uint4 wb = *reinterpret_cast<const uint4*>(sb + (g + 8) * kBulkRowBytes + c * 64 + t4 * 16);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)(nt * 8 + g) * KP + c * 32 + 8 * t4);
              mma_bf16_16816(acc[nt], wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
              mma_bf16_16816(acc[nt], wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[slot]);
      ++it;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        float* pr = red + (size_t)warp * 256;
        *reinterpret_cast<float2*>(pr + g * 16 + nt * 8 + 2 * t4) = make_float2(acc[nt][0], acc[nt][1]);
        *reinterpret_cast<float2*>(pr + (g + 8) * 16 + nt * 8 + 2 * t4) = make_float2(acc[nt][2], acc[nt][3]);
      }
      csync_bulk();
      {
        const int r = tid >> 4, col = tid & 15;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) s += red[w * 256 + r * 16 + col];
        tile_out[r * 17 + col] = s;
      }
      csync_bulk();
      {  // store: rows [0, d) -> v0, [d, 2d) -> A, [2d, 3d) -> B_hist[:, t]
        const int r = tid >> 4, b = tid & 15;
        const int n = tile * 16 + r, seg = n / d, c = n - seg * d;
        if (n < 3 * d && b < batch && !*reinterpret_cast<volatile int*>(&sh->abort)) {
          const __nv_bfloat16 v = f2bf(tile_out[r * 17 + b]);
          if (seg == 0) p.v0[(size_t)b * d + c] = v;
          else if (seg == 1) p.a[(size_t)b * d + c] = v;
          else p.bh[((size_t)b * p.max_len + t) * d + c] = v;
        }
      }
    }
    if (tile < a_lo || tile >= a_hi) continue;
    {  // ---- the gate readouts' share of these 16 columns of A
      const int k0 = tile * 16 - d;
      for (int i = tid; i < batch * p.L * 16; i += kTcWarps * 32) {
        const int b = i / (p.L * 16), rem = i - b * (p.L * 16), l = rem >> 4, kk = rem & 15;
        const int src = t - (1 << l);
        bool ok = src >= 0;
        if (ok && p.doc) ok = p.doc[(size_t)b * p.max_len + src] == p.doc[(size_t)b * p.max_len + t];
        const float av = bf2f(f2bf(tile_out[kk * 17 + b]));  // A as stored (bf16)
        const float bs = ok ? bf2f(p.bh[((size_t)b * p.max_len + src) * d + k0 + kk]) : 0.f;
        const float h = fmaxf(av + bs, 0.f);
        hv[(b * kGateMaxL + l) * 16 + kk] = h * h;  // relu squared
      }
      csync_bulk();
      const int slot = it % nslots;
      bool ok = !*reinterpret_cast<volatile int*>(&sh->abort);
      if (ok && !mbar_wait(&sh->full[slot], (uint32_t)((it / nslots) & 1), status, wait_limit)) {
        sh->abort = 1;
        ok = false;
      }
      if (ok) {
        const __nv_bfloat16* wg = reinterpret_cast<const __nv_bfloat16*>(slots + (size_t)slot * kBulkSlotBytes);
        for (int o = tid; o < LNP; o += kTcWarps * 32) {
          const int l = o / p.NP;
          if (o - l * p.NP >= p.H3) continue;  // padding rows of the packed gates
          float w[16];
#pragma unroll
          for (int kk = 0; kk < 16; ++kk) w[kk] = bf2f(wg[(size_t)kk * LNP + o]);
          for (int b = 0; b < batch; ++b) {
            const float* hb = hv + (b * kGateMaxL + l) * 16;
            float s = 0.f;
#pragma unroll
            for (int kk = 0; kk < 16; ++kk) s = fmaf(w[kk], hb[kk], s);
            atomicAdd(p.pre + (size_t)b * LNP + o, s);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[slot]);
      ++it;
    }
  }
}

// ---------------------------------------------------------------- attention
struct AttnParams {
  const __nv_bfloat16 *q, *k, *v;
  __nv_bfloat16* y;
  const int64_t* t_buf;
  float* part;
  int* counters;
  int max_len, H, window, chunk_cap;
};

__device__ __forceinline__ float block_reduce_128(float v, float* sred, bool is_max) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = is_max ? warp_max(v) : warp_sum(v);
  __syncthreads();
  if (lane == 0) sred[warp] = v;
  __syncthreads();
  float r = sred[0];
#pragma unroll
  for (int w = 1; w < 4; ++w) r = is_max ? fmaxf(r, sred[w]) : r + sred[w];
  return r;
}

// grid (H, batch, nsplit), 128 threads, hd = 64.
__global__ void __launch_bounds__(128) attn_decode_kernel(AttnParams p) {
  constexpr int HD = 64;
  extern __shared__ float sc[];  // [chunk_cap]
  __shared__ float sq[HD];
  __shared__ float sred[4];
  __shared__ float sacc[16][HD];
  __shared__ int s_last;
  const int h = blockIdx.x, b = blockIdx.y, split = blockIdx.z, nsplit = gridDim.z;
  const int tid = threadIdx.x;
  const int H = p.H, d = H * HD;
  pdl_trigger();
  const long long t = *p.t_buf;
  const long long lo = p.window > 0 ? (t + 1 - p.window > 0 ? t + 1 - p.window : 0) : 0;
  const long long n = t + 1 - lo;
  const long long chunk = (n + nsplit - 1) / nsplit;
  const long long s0 = lo + split * chunk;
  long long s1 = s0 + chunk;
  if (s1 > t + 1) s1 = t + 1;
  const int cnt = s1 > s0 ? (int)(s1 - s0) : 0;
  // cache rows before t were written by earlier steps: the blocks of head 0
  // warm whole rows (every head, 2 KB each) into L2 for the blocks of all
  // heads (one bulk prefetch per row, not one per 128-byte head slice)
  if (h == 0) {
    for (int i = tid; i < cnt; i += 128) {
      if (s0 + i < t) {
        prefetch_l2(p.k + ((size_t)b * p.max_len + s0 + i) * d, (uint32_t)d * 2);
        prefetch_l2(p.v + ((size_t)b * p.max_len + s0 + i) * d, (uint32_t)d * 2);
      }
    }
  }
  pdl_wait();
  if (tid < HD) sq[tid] = bf2f(p.q[(size_t)b * d + h * HD + tid]);
  __syncthreads();
  const float scale = rsqrtf((float)HD);

  // scores: eight lanes per key row (its 128 bytes read coalesced), partial
  // dot products joined by three shuffles, eight rows in flight per thread;
  // every lane runs the same rounds, so the shuffles see whole warps
  const int kg = tid & 7, rs = tid >> 3;  // 16 row groups of 8 lanes
  float qf[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) qf[e] = sq[kg * 8 + e];
  float mloc = -INFINITY;
  for (int base = 0; base < cnt; base += 128) {
    uint4 kv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + rs + 16 * u;
      kv[u] = i < cnt ? *reinterpret_cast<const uint4*>(p.k + ((size_t)b * p.max_len + s0 + i) * d +
                                                         h * HD + kg * 8)
                      : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + rs + 16 * u;
      float f[8];
      unpack8(kv[u], f);
      float sd = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) sd = fmaf(f[e], qf[e], sd);
      sd += __shfl_xor_sync(0xffffffffu, sd, 1);
      sd += __shfl_xor_sync(0xffffffffu, sd, 2);
      sd += __shfl_xor_sync(0xffffffffu, sd, 4);
      if (i < cnt) {
        sd *= scale;
        if (kg == 0) sc[i] = sd;
        mloc = fmaxf(mloc, sd);
      }
    }
  }
  const float M = block_reduce_128(mloc, sred, true);
  float lsum = 0.f;
  for (int i = tid; i < cnt; i += 128) {
    const float e = expf(sc[i] - M);
    sc[i] = e;
    lsum += e;
  }
  const float Lsum = block_reduce_128(lsum, sred, false);  // includes a barrier after sc writes
  // values: thread (row group r, channel group cg) accumulates channels
  // [8 cg, +8) over positions r, r + 16, ...; eight 16-byte rows in flight
  const int cg = tid & 7, r0 = tid >> 3;
  float acc8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) acc8[e] = 0.f;
  for (int i0 = r0; i0 < cnt; i0 += 128) {
    uint4 vv[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + 16 * u;
      if (i < cnt)
        vv[u] = *reinterpret_cast<const uint4*>(p.v + ((size_t)b * p.max_len + s0 + i) * d + h * HD + cg * 8);
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = i0 + 16 * u;
      if (i < cnt) {
        float f[8];
        unpack8(vv[u], f);
        const float w = sc[i];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc8[e] = fmaf(w, f[e], acc8[e]);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) sacc[r0][cg * 8 + e] = acc8[e];
  __syncthreads();
  float o = 0.f;
  if (tid < HD) {
#pragma unroll
    for (int r = 0; r < 16; ++r) o += sacc[r][tid];
  }
  if (nsplit == 1) {
    if (tid < HD) p.y[(size_t)b * d + h * HD + tid] = f2bf(cnt > 0 ? o / Lsum : 0.f);
    return;
  }
  float* mine = p.part + (((size_t)b * H + h) * nsplit + split) * (HD + 2);
  if (tid < HD) mine[2 + tid] = o;
  if (tid == 0) {
    mine[0] = cnt > 0 ? M : -INFINITY;
    mine[1] = cnt > 0 ? Lsum : 0.f;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(&p.counters[b * H + h], 1) == nsplit - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float* all = p.part + ((size_t)b * H + h) * nsplit * (HD + 2);
  float Mx = -INFINITY;
  for (int s = 0; s < nsplit; ++s) Mx = fmaxf(Mx, __ldcg(all + s * (HD + 2)));
  if (tid < HD) {
    float num = 0.f, den = 0.f;
    for (int s = 0; s < nsplit; ++s) {
      const float ms = __ldcg(all + s * (HD + 2));
      if (ms == -INFINITY) continue;
      const float w = expf(ms - Mx);
      den += w * __ldcg(all + s * (HD + 2) + 1);
      num += w * __ldcg(all + s * (HD + 2) + 2 + tid);
    }
    p.y[(size_t)b * d + h * HD + tid] = f2bf(den > 0.f ? num / den : 0.f);
  }
  if (tid == 0) p.counters[b * H + h] = 0;
}

// ---------------------------------------------------------------- fused FFN
// h = RMSNorm(x_in); u = silu(h . Wg^T) * (h . Wu^T) (bf16); x += u . Wd^T.
// One launch instead of two: CTA c owns a contiguous run of u elements,
// forms them as the SwiGLU GEMV does (warp per unit, transpose-reduction over
// the lockstep rows), keeps them in shared memory and adds their share of the
// down projection, rows of Wd^T (ff x d, contiguous per u element), into the
// fp32 residual x with vector atomics.  x_in is a copy of x written by the
// preceding residual kernel, so no block reads x while others add into it.
struct FfnParams {
  const float* x_in;
  const __nv_bfloat16* norm_w;
  const __nv_bfloat16 *wg, *wu, *wdT;
  float* x;
  int d, ff, batch, upc;  // upc: u elements per CTA
};

constexpr int kFfnMaxUpc = 32;

__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

constexpr int kFfnWarps = 16;
constexpr int kFfnMaxK = 2048;  // d supported by the fully unrolled row loop

template <int MAXB>
__global__ void __launch_bounds__(kFfnWarps * 32) ffn_kernel(FfnParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(smem_raw);  // [batch][d]
  __shared__ float s_rstd[MAXB];
  __shared__ float us[MAXB][kFfnMaxUpc];
  pdl_trigger();
  const int d = p.d, batch = p.batch;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int u0 = blockIdx.x * p.upc;
  const int u1 = min(p.ff, u0 + p.upc);
  // weights do not depend on the previous kernel: warm them into L2
  for (int u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
    prefetch_l2(p.wg + (size_t)u * d, (uint32_t)d * 2);
    prefetch_l2(p.wu + (size_t)u * d, (uint32_t)d * 2);
    prefetch_l2(p.wdT + (size_t)u * d, (uint32_t)d * 2);
  }
  pdl_wait();

  // normalised input rows in shared memory (bf16).  Up to 4 rows: one pass,
  // every thread keeps its float4s of the rows in registers and the squares
  // are reduced per row in shared memory; more rows: a warp per row sums,
  // then all threads scale.
  if constexpr (MAXB <= 4) {
    const int k4 = d / 4, n4 = batch * k4;
    if (threadIdx.x < MAXB) s_rstd[threadIdx.x] = 0.f;  // sums accumulate below
    __syncthreads();
    constexpr int NV = (MAXB * kFfnMaxK / 4 + kFfnWarps * 32 - 1) / (kFfnWarps * 32);
    float4 v[NV];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * kFfnWarps * 32;
      float sq = 0.f;
      if (i < n4) {
        v[j] = reinterpret_cast<const float4*>(p.x_in)[i];
        sq = v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
      }
      if ((k4 & 31) == 0) {  // a warp's 32 float4s lie in one row: reduce first
        sq = warp_sum(sq);
        if (lane == 0 && i < n4) atomicAdd(&s_rstd[i / k4], sq);
      } else if (i < n4) {
        atomicAdd(&s_rstd[i / k4], sq);
      }
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const int i = threadIdx.x + j * kFfnWarps * 32;
      if (i < n4) {
        const int b = i / k4, k = (i - b * k4) * 4;
        const float r = rsqrtf(s_rstd[b] / (float)d + kNormEps);
        uint2 pk;
        pk.x = pack2(v[j].x * r * bf2f(p.norm_w[k]), v[j].y * r * bf2f(p.norm_w[k + 1]));
        pk.y = pack2(v[j].z * r * bf2f(p.norm_w[k + 2]), v[j].w * r * bf2f(p.norm_w[k + 3]));
        *reinterpret_cast<uint2*>(xs + (size_t)b * d + k) = pk;
      }
    }
  } else {
    for (int b = warp; b < batch; b += kFfnWarps) {
      const float4* xr = reinterpret_cast<const float4*>(p.x_in + (size_t)b * d);
      float ss = 0.f;
      for (int i = lane; i < d / 4; i += 32) {
        const float4 v = xr[i];
        ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
      }
      ss = warp_sum(ss);
      if (lane == 0) s_rstd[b] = rsqrtf(ss / (float)d + kNormEps);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < batch * d / 4; i += blockDim.x) {
      const int b = i / (d / 4), k = (i - b * (d / 4)) * 4;
      const float4 v = reinterpret_cast<const float4*>(p.x_in + (size_t)b * d)[k / 4];
      const float r = s_rstd[b];
      uint2 pk;
      pk.x = pack2(v.x * r * bf2f(p.norm_w[k]), v.y * r * bf2f(p.norm_w[k + 1]));
      pk.y = pack2(v.z * r * bf2f(p.norm_w[k + 2]), v.w * r * bf2f(p.norm_w[k + 3]));
      *reinterpret_cast<uint2*>(xs + (size_t)b * d + k) = pk;
    }
  }
  __syncthreads();

  // u elements of this CTA: warp per element, gate and up rows together; the
  // whole row pair is requested at once (one round trip per element)
  for (int u = u0 + warp; u < u1; u += kFfnWarps) {
    const __nv_bfloat16* r0 = p.wg + (size_t)u * d;
    const __nv_bfloat16* r1 = p.wu + (size_t)u * d;
    float acc[2 * MAXB];
#pragma unroll
    for (int i = 0; i < 2 * MAXB; ++i) acc[i] = 0.f;
    auto fma_chunk = [&](const uint4& ua, const uint4& ub, int k) {
      float fa[8], fb[8];
      unpack8(ua, fa);
      unpack8(ub, fb);
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        if (b < batch) {
          float fx[8];
          unpack8(*reinterpret_cast<const uint4*>(xs + (size_t)b * d + k), fx);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            acc[b] = fmaf(fa[j], fx[j], acc[b]);
            acc[MAXB + b] = fmaf(fb[j], fx[j], acc[MAXB + b]);
          }
        }
      }
    };
    if constexpr (MAXB <= 4) {
      // the whole row pair requested at once: one round trip per element
      constexpr int KI = kFfnMaxK / 256;
      uint4 wa[KI], wb[KI];
#pragma unroll
      for (int i = 0; i < KI; ++i) {
        const int k = lane * 8 + i * 256;
        if (k < d) {
          wa[i] = ld_stream16(r0 + k);
          wb[i] = ld_stream16(r1 + k);
        }
      }
#pragma unroll
      for (int i = 0; i < KI; ++i) {
        const int k = lane * 8 + i * 256;
        if (k < d) fma_chunk(wa[i], wb[i], k);
      }
    } else {
#pragma unroll 2
      for (int k = lane * 8; k < d; k += 256) fma_chunk(ld_stream16(r0 + k), ld_stream16(r1 + k), k);
    }
    const float rr = transpose_reduce<2 * MAXB>(acc);
    const float other = __shfl_xor_sync(0xffffffffu, rr, MAXB);
    const int b = lane % MAXB, row = (lane / MAXB) & 1;
    if (lane < 2 * MAXB && row == 0 && b < batch) {
      const float g = rr, up = other;
      us[b][u - u0] = bf2f(f2bf(g / (1.0f + expf(-g)) * up));  // u in bf16, as the reference
    }
  }
  __syncthreads();

  // this CTA's share of the down projection: x[b, o] += sum_j Wd^T[u0 + j, o] * u[b, j]
  const int nu = u1 - u0;
  for (int o = threadIdx.x * 4; o < d; o += blockDim.x * 4) {
    float acc[MAXB][4];
#pragma unroll
    for (int b = 0; b < MAXB; ++b) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
    auto fma_row = [&](const uint2& w2, int j) {
      const float2 wa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w2.x));
      const float2 wb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w2.y));
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
        if (b < batch) {
          const float uv = us[b][j];
          acc[b][0] = fmaf(wa.x, uv, acc[b][0]);
          acc[b][1] = fmaf(wa.y, uv, acc[b][1]);
          acc[b][2] = fmaf(wb.x, uv, acc[b][2]);
          acc[b][3] = fmaf(wb.y, uv, acc[b][3]);
        }
      }
    };
    if constexpr (MAXB <= 4) {  // every row requested at once
      uint2 w[kFfnMaxUpc];
#pragma unroll
      for (int j = 0; j < kFfnMaxUpc; ++j)
        if (j < nu) w[j] = __ldg(reinterpret_cast<const uint2*>(p.wdT + (size_t)(u0 + j) * d + o));
#pragma unroll
      for (int j = 0; j < kFfnMaxUpc; ++j)
        if (j < nu) fma_row(w[j], j);
    } else {
#pragma unroll 4
      for (int j = 0; j < nu; ++j)
        fma_row(__ldg(reinterpret_cast<const uint2*>(p.wdT + (size_t)(u0 + j) * d + o)), j);
    }
#pragma unroll
    for (int b = 0; b < MAXB; ++b)
      if (b < batch) red_add_v4(p.x + (size_t)b * d + o, acc[b][0], acc[b][1], acc[b][2], acc[b][3]);
  }
}

// ---------------------------------------------------------------- fused FFN, bulk copies
// The whole FFN (up to 16 lockstep rows per launch, d <= 1024) with the
// weights through the copy engine: CTA c takes tiles of 8 u elements (16
// rows: gate and up row of each element, the tensor-core GEMV tile above)
// and, as the next ring item of each tile, the 8 matching rows of Wd^T.  A producer warp issues every copy
// it can before the dependency wait; the consumers stage RMSNorm(x_in),
// form u = silu(gate) * up (rounded to bf16) per tile, fold u into this
// CTA's down-projection partials (registers, 4 output columns per thread),
// and add the partials into x once at the end (vector reductions).
template <int MAXB>
__global__ void __launch_bounds__(kBulkThreads, 1)
    ffn_bulk_kernel(FfnParams p, int nslots, int* status, uint32_t wait_limit) {
  constexpr int NT = MAXB > 8 ? 2 : 1;  // 8-column mma tiles of lockstep rows
  extern __shared__ __align__(128) unsigned char ffn_smem[];
  const int d = p.d, batch = p.batch, KP = d + 32, ff = p.ff;
  uint8_t* slots = ffn_smem;                                                     // [nslots][16][2112]
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(ffn_smem + (size_t)nslots * kBulkSlotBytes);
  float* red = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(xs) + bulk_xs_bytes(NT, d));
  float* tile_out = red + kTcWarps * 16 * 16;   // [16][17]
  float* us = tile_out + 16 * 17;               // [MAXB][8]
  BulkShared* sh = reinterpret_cast<BulkShared*>(us + MAXB * 8);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ntiles = (ff + 7) / 8;
  const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int nitems = 2 * my_tiles;  // (gate/up tile, Wd^T rows) per tile
  if (tid == 0) {
    for (int i = 0; i < nslots; ++i) {
      mbar_init(&sh->full[i], 1);
      mbar_init(&sh->empty[i], kTcWarps);
    }
    sh->abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  pdl_trigger();

  if (warp == kTcWarps) {  // ---------------- producer (one lane)
    if (lane != 0) return;
    int issued = 0;
    for (int item = 0; item < nitems; ++item) {
      const int slot = item % nslots;
      if (item >= nslots &&
          !mbar_wait(&sh->empty[slot], (uint32_t)(((item / nslots) - 1) & 1), status, wait_limit)) {
        sh->abort = 1;
        break;
      }
      if (*reinterpret_cast<volatile int*>(&sh->abort)) break;
      const int tile = blockIdx.x + (item >> 1) * gridDim.x;
      uint8_t* dst = slots + (size_t)slot * kBulkSlotBytes;
      const int nrows = (item & 1) ? 8 : 16;
      mbar_arrive_expect_tx(&sh->full[slot], (uint32_t)(nrows * d * 2));
      for (int r = 0; r < nrows; ++r) {
        const __nv_bfloat16* row;
        if (item & 1) {
          row = p.wdT + (size_t)min(tile * 8 + r, ff - 1) * d;
        } else {
          const int u = min(tile * 8 + (r >> 1), ff - 1);
          row = ((r & 1) ? p.wu : p.wg) + (size_t)u * d;
        }
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                smem_u32(dst + r * kBulkRowBytes)),
            "l"(row), "r"((uint32_t)(d * 2)), "r"(smem_u32(&sh->full[slot]))
            : "memory");
      }
      ++issued;
    }
    for (int sl = 0; sl < nslots; ++sl) {  // nothing in flight into this CTA when it exits
      const int n_s = issued / nslots + (sl < issued % nslots ? 1 : 0);
      if (n_s > 0) mbar_wait(&sh->full[sl], (uint32_t)((n_s - 1) & 1), nullptr, 1u << 20);
    }
    return;
  }

  // ---------------- consumers (8 warps, named barrier 1)
  const int g = lane >> 2, t4 = lane & 3;
  pdl_wait();
  for (int rb = warp; rb < batch; rb += kTcWarps) {  // RMSNorm(x_in) rows as bf16, warp per row
    const int k4 = d / 4;
    {
      const float* xr = p.x_in + (size_t)rb * d;
      float4 v[8];
      uint2 wn[8];
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < k4 ? reinterpret_cast<const float4*>(xr)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
        wn[j] = i < k4 ? *reinterpret_cast<const uint2*>(p.norm_w + 4 * i) : make_uint2(0, 0);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
      const float sc = rsqrtf(warp_sum(ss) / (float)d + kNormEps);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int i = lane + 32 * j;
        if (i < k4) {
          const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wn[j].x));
          const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wn[j].y));
          uint2 pk;
          pk.x = pack2(v[j].x * sc * w01.x, v[j].y * sc * w01.y);
          pk.y = pack2(v[j].z * sc * w23.x, v[j].w * sc * w23.y);
          *reinterpret_cast<uint2*>(xs + (size_t)rb * KP + 4 * i) = pk;
        }
      }
    }
  }
  csync_bulk();

  const int o = 4 * tid;  // this thread's 4 output columns of the down projection
  float dacc[MAXB][4];
#pragma unroll
  for (int b = 0; b < MAXB; ++b) dacc[b][0] = dacc[b][1] = dacc[b][2] = dacc[b][3] = 0.f;
  const int nchunks = d / 32;
  for (int item = 0; item < nitems; ++item) {
    const int slot = item % nslots;
    const int tile = blockIdx.x + (item >> 1) * gridDim.x;
    bool ok = !*reinterpret_cast<volatile int*>(&sh->abort);
    if (ok && !mbar_wait(&sh->full[slot], (uint32_t)((item / nslots) & 1), status, wait_limit)) {
      sh->abort = 1;
      ok = false;
    }
    const uint8_t* sb = slots + (size_t)slot * kBulkSlotBytes;
    if ((item & 1) == 0) {  // gate/up tile -> u of its 8 elements
      float acc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
      if (ok) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = warp * 4 + i;
          if (c < nchunks) {
            const uint4 wa = *reinterpret_cast<const uint4*>(sb + g * kBulkRowBytes + c * 64 + t4 * 16);
            const uint4 wb = *reinterpret_cast<const uint4*>(sb + (g + 8) * kBulkRowBytes + c * 64 + t4 * 16);
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
              const uint4 xv = *reinterpret_cast<const uint4*>(xs + (size_t)(nt * 8 + g) * KP + c * 32 + 8 * t4);
              mma_bf16_16816(acc[nt], wa.x, wb.x, wa.y, wb.y, xv.x, xv.y);
              mma_bf16_16816(acc[nt], wa.z, wb.z, wa.w, wb.w, xv.z, xv.w);
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[slot]);
      float* pr = red + (size_t)warp * 256;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        *reinterpret_cast<float2*>(pr + g * 16 + nt * 8 + 2 * t4) = make_float2(acc[nt][0], acc[nt][1]);
        *reinterpret_cast<float2*>(pr + (g + 8) * 16 + nt * 8 + 2 * t4) = make_float2(acc[nt][2], acc[nt][3]);
      }
      csync_bulk();
      {  // rows 0..15, columns (lockstep rows) 0..15
        const int r = tid >> 4, col = tid & 15;
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kTcWarps; ++w) s += red[w * 256 + r * 16 + col];
        tile_out[r * 17 + col] = s;
      }
      csync_bulk();
      if (tid < 8 * MAXB) {  // tile row 2j = gate of element j, 2j + 1 = its up row
        const int j = tid / MAXB, b = tid - j * MAXB;
        const float gt = tile_out[(2 * j) * 17 + b], up = tile_out[(2 * j + 1) * 17 + b];
        const bool live = b < batch && tile * 8 + j < ff;
        us[b * 8 + j] = live ? bf2f(f2bf(gt / (1.0f + expf(-gt)) * up)) : 0.f;  // u in bf16
      }
      csync_bulk();
    } else {  // Wd^T rows of the same 8 elements: this CTA's share of x += u . Wd^T
      if (ok && o < d) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint2 w2 = *reinterpret_cast<const uint2*>(sb + j * kBulkRowBytes + o * 2);
          const float2 wa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w2.x));
          const float2 wb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w2.y));
#pragma unroll
          for (int b = 0; b < MAXB; ++b) {
            const float uv = us[b * 8 + j];
            dacc[b][0] = fmaf(wa.x, uv, dacc[b][0]);
            dacc[b][1] = fmaf(wa.y, uv, dacc[b][1]);
            dacc[b][2] = fmaf(wb.x, uv, dacc[b][2]);
            dacc[b][3] = fmaf(wb.y, uv, dacc[b][3]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh->empty[slot]);
    }
  }
  if (my_tiles > 0 && o < d && !*reinterpret_cast<volatile int*>(&sh->abort)) {
#pragma unroll
    for (int b = 0; b < MAXB; ++b)
      if (b < batch) red_add_v4(p.x + (size_t)b * d + o, dacc[b][0], dacc[b][1], dacc[b][2], dacc[b][3]);
  }
}

// ---------------------------------------------------------------- small ones
__global__ void embed_kernel(const int64_t* tokens, const __nv_bfloat16* emb, float* x, int d,
                             int vocab, int* status) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x;
  long long tok = tokens[b];
  if (tok < 0 || tok >= vocab) {
    if (status && threadIdx.x == 0) atomicExch(status, 1);
    tok = tok < 0 ? 0 : vocab - 1;
  }
  for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
    float f[8];
    unpack8(*reinterpret_cast<const uint4*>(emb + (size_t)tok * d + c), f);
    float4* xo = reinterpret_cast<float4*>(x + (size_t)b * d + c);
    xo[0] = make_float4(f[0], f[1], f[2], f[3]);
    xo[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

// document id of the position being decoded: the previous position's id,
// plus one if the previous token was the separator (exclusive cumulative
// count of separators, the forward's doc_id)
__global__ void doc_step_kernel(const int64_t* tokens, const int64_t* t_buf, int* doc,
                                int64_t* last_tok, int64_t eot, int max_len, int batch) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const long long t = *t_buf;
  if (t < 0 || t >= max_len) return;
  const int id = t > 0 ? doc[(size_t)b * max_len + t - 1] + (last_tok[b] == eot ? 1 : 0) : 0;
  doc[(size_t)b * max_len + t] = id;
  last_tok[b] = tokens[b];
}

// Greedy token choice on the device: one block per row, the first index of
// the row's largest logit (torch.argmax's tie rule; the logits are the
// step's bf16 values), written to the next step's input and to an output
// vector.
__global__ void __launch_bounds__(1024) argmax_kernel(const __nv_bfloat16* logits, int vocab,
                                                      int64_t* next_tokens, int64_t* out) {
  __shared__ float s_v[32];
  __shared__ int s_i[32];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const __nv_bfloat16* row = logits + (size_t)b * vocab;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < vocab; i += 1024) {  // ascending per thread: the first max is kept
    const float v = bf2f(row[i]);
    if (v > best) {
      best = v;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    s_v[warp] = best;
    s_i[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = s_v[lane];
    bi = s_i[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      const int64_t tok = bi == 0x7fffffff ? 0 : bi;  // an all-NaN row picks 0
      next_tokens[b] = tok;
      if (out) out[b] = tok;
    }
  }
}

// Top-k / temperature sampling on the device, one block per row: the k-th
// largest logit by a two-pass radix select over the bf16 keys, then a draw
// from softmax(logit / T) restricted to the logits >= that value (the
// reference's rule, modeling_dispatcher.py:427-432: every logit below the
// k-th largest masked, ties at it kept) as the Gumbel-max over those
// candidates.  The uniforms come from a counter-based hash of (seed,
// position t, row, index): a fresh draw every step with no generator state.
__device__ __forceinline__ uint32_t bf16_key(__nv_bfloat16 v) {  // order-preserving
  const uint16_t u = *reinterpret_cast<const uint16_t*>(&v);
  return (u & 0x8000u) ? (uint32_t)(uint16_t)~u : (uint32_t)(u | 0x8000u);
}

__device__ __forceinline__ uint64_t mix64(uint64_t z) {  // splitmix64 finaliser
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// bin of the 256-bin histogram (from the top) that holds the k-th largest
// key, and the number of keys in the bins above it
__device__ __forceinline__ void select_bin(const int* hist, int k, int& bin, int& above) {
  __shared__ int s_bin, s_above;
  if (threadIdx.x == 0) {
    int acc = 0, bsel = 0;
    for (int j = 255; j >= 0; --j) {
      if (acc + hist[j] >= k) {
        bsel = j;
        break;
      }
      acc += hist[j];
    }
    s_bin = bsel;
    s_above = acc;
  }
  __syncthreads();
  bin = s_bin;
  above = s_above;
}

__global__ void __launch_bounds__(1024) sample_top_k_kernel(const __nv_bfloat16* logits, int vocab,
                                                            int k, float inv_temp,
                                                            unsigned long long seed,
                                                            const int64_t* t_buf,
                                                            int64_t* next_tokens, int64_t* out) {
  __shared__ int hist[256];
  __shared__ float s_v[32];
  __shared__ int s_i[32];
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const __nv_bfloat16* row = logits + (size_t)b * vocab;
  const int kk = k < 1 ? 1 : (k > vocab ? vocab : k);
  // pass 1: high byte of the key
  for (int j = tid; j < 256; j += 1024) hist[j] = 0;
  __syncthreads();
  for (int i = tid; i < vocab; i += 1024) atomicAdd(&hist[bf16_key(row[i]) >> 8], 1);
  __syncthreads();
  int hi, above_hi;
  select_bin(hist, kk, hi, above_hi);
  __syncthreads();
  // pass 2: low byte among the keys of that high byte
  for (int j = tid; j < 256; j += 1024) hist[j] = 0;
  __syncthreads();
  for (int i = tid; i < vocab; i += 1024) {
    const uint32_t key = bf16_key(row[i]);
    if ((int)(key >> 8) == hi) atomicAdd(&hist[key & 255], 1);
  }
  __syncthreads();
  int lo, above_lo;
  select_bin(hist, kk - above_hi, lo, above_lo);
  const uint32_t thr = ((uint32_t)hi << 8) | (uint32_t)lo;  // key of the k-th largest logit
  // Gumbel-max over the candidates
  const uint64_t base = mix64(seed ^ mix64((uint64_t)*t_buf * 0x9e3779b97f4a7c15ull + (uint64_t)b));
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < vocab; i += 1024) {
    const __nv_bfloat16 v = row[i];
    if (bf16_key(v) < thr) continue;
    const uint64_t h = mix64(base + (uint64_t)i);
    const float u = ((float)(uint32_t)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);  // in (0, 1)
    const float z = bf2f(v) * inv_temp - logf(-logf(u));
    if (z > best) {
      best = z;
      bi = i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) {
      best = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    s_v[warp] = best;
    s_i[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    best = s_v[lane];
    bi = s_i[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      const int64_t tok = bi == 0x7fffffff ? 0 : bi;
      next_tokens[b] = tok;
      if (out) out[b] = tok;
    }
  }
}

__global__ void advance_kernel(int64_t* t) {
  pdl_trigger();
  pdl_wait();
  t[0] += 1;
}

}  // namespace
}  // namespace dh

using namespace dh;

#define BF(p) reinterpret_cast<const __nv_bfloat16*>(p)
#define BFM(p) reinterpret_cast<__nv_bfloat16*>(p)
#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

extern "C" int dh_decode_embed(const int64_t* tokens, const void* emb, float* x, int batch, int d,
                               int vocab, int* status, void* stream) {
  DH_REQUIRE(tokens && emb && x, DH_ERR_ARG, "dh_decode_embed: null pointer");
  DH_REQUIRE(batch > 0 && d % 8 == 0 && vocab > 0, DH_ERR_SHAPE, "dh_decode_embed: bad sizes");
  if (launch_pdl(embed_kernel, dim3(batch), dim3(128), 0, STREAM(stream), tokens, BF(emb), x, d,
                 vocab, status))
    return check_launch("embed_kernel");
  return DH_OK;
}

extern "C" int dh_decode_mixer_in(const float* x, const void* norm_w, const void* w3, void* v0,
                                  void* a_out, void* b_hist, const int64_t* t_buf, int max_len,
                                  int batch, int d, int* status, void* stream) {
  DH_REQUIRE(x && norm_w && w3 && v0 && a_out && b_hist && t_buf, DH_ERR_ARG,
             "dh_decode_mixer_in: null pointer");
  DH_REQUIRE(d % 8 == 0 && max_len > 0, DH_ERR_SHAPE, "dh_decode_mixer_in: bad sizes");
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    GemvIn in{x + (size_t)b0 * d, 1, BF(norm_w), d, nb, status};
    EpiMixerIn e{BF(w3), d, d, max_len, BFM(v0) + (size_t)b0 * d, BFM(a_out) + (size_t)b0 * d,
                 BFM(b_hist) + (size_t)b0 * max_len * d, t_buf};
    int rc = launch_gemv(in, e, 3 * d / 2, STREAM(stream));
    if (rc) return rc;
  }
  return DH_OK;
}

extern "C" int dh_decode_tree_step(const void* a_in, const void* b_hist, const void* wi,
                                   const void* wf, const void* wr, const float* bi,
                                   const float* bf, const float* br, const int64_t* t_buf,
                                   float* ig, float* fg, void* rg_hist, const void* v0,
                                   void* v_ring, void* y, int* counters, const int* doc_hist,
                                   int batch, int max_len, int L, int H, int hd, int gh,
                                   void* stream) {
  DH_REQUIRE(a_in && b_hist && wi && wf && wr && bi && bf && br && t_buf && ig && fg && rg_hist &&
                 v0 && v_ring && y && counters,
             DH_ERR_ARG, "dh_decode_tree_step: null pointer");
  DH_REQUIRE(L >= 1 && L <= 16 && H >= 1 && hd % 8 == 0 && hd <= 8 * kTreeGroups &&
                 gh % 8 == 0 && batch > 0,
             DH_ERR_SHAPE, "dh_decode_tree_step: bad sizes (L=%d H=%d hd=%d gh=%d)", L, H, hd, gh);
  const int d = H * hd, S = (1 << (L + 1)) - 2;
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    TreeStepParams p{BF(a_in) + (size_t)b0 * gh,
                     BF(b_hist) + (size_t)b0 * max_len * gh,
                     BF(wi), BF(wf), BF(wr), bi, bf, br, t_buf,
                     ig + (size_t)b0 * L * H, fg + (size_t)b0 * L * H,
                     BFM(rg_hist) + (size_t)b0 * max_len * L * H,
                     BF(v0) + (size_t)b0 * d,
                     BFM(v_ring) + (size_t)b0 * S * d,
                     BFM(y) + (size_t)b0 * d,
                     counters, doc_hist ? doc_hist + (size_t)b0 * max_len : nullptr,
                     nb, max_len, L, H, hd, gh, S};
    dim3 grid(L, H);
    const int bad = nb == 1   ? launch_pdl(tree_step_kernel<1>, grid, dim3(128), 0, STREAM(stream), p)
                    : nb <= 4 ? launch_pdl(tree_step_kernel<4>, grid, dim3(128), 0, STREAM(stream), p)
                              : launch_pdl(tree_step_kernel<16>, grid, dim3(128), 0, STREAM(stream), p);
    if (bad) return check_launch("tree_step_kernel");
  }
  return DH_OK;
}

extern "C" int dh_decode_tree_step_tc(const void* a_in, const void* b_hist, const void* w_gates,
                                      int np, const float* bi, const float* bf, const float* br,
                                      const int64_t* t_buf, float* pre, void* rg_hist,
                                      const void* v0, void* v_ring, void* y, const int* doc_hist,
                                      int batch, int max_len, int L, int H, int hd, int gh,
                                      void* stream) {
  DH_REQUIRE(a_in && b_hist && w_gates && bi && bf && br && t_buf && pre && rg_hist && v0 &&
                 v_ring && y,
             DH_ERR_ARG, "dh_decode_tree_step_tc: null pointer");
  DH_REQUIRE(L >= 1 && L <= 16 && H >= 1 && np % 16 == 0 && np >= 3 * H && np <= 48 &&
                 hd >= 1 && hd <= 64 && gh % 32 == 0 && batch >= 1,
             DH_ERR_SHAPE, "dh_decode_tree_step_tc: unsupported sizes (L=%d H=%d np=%d hd=%d gh=%d)",
             L, H, np, hd, gh);
  DH_REQUIRE(aligned16(a_in) && aligned16(b_hist) && aligned16(w_gates), DH_ERR_ARG,
             "dh_decode_tree_step_tc: a, B_hist and the gate weights must be 16-byte aligned");
  const int d = H * hd, S = (1 << (L + 1)) - 2;
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    const int* doc = doc_hist ? doc_hist + (size_t)b0 * max_len : nullptr;
    float* pr = pre + (size_t)b0 * L * np;
    TreeGatesTcParams gp{BF(a_in) + (size_t)b0 * gh, BF(b_hist) + (size_t)b0 * max_len * gh,
                         BF(w_gates), t_buf, doc, pr, BF(v_ring) + (size_t)b0 * S * d, nb,
                         max_len, L, np, gh, S, d};
    const dim3 gg(L, (gh + 255) / 256);
    const int bad = np <= 16   ? launch_pdl(tree_gates_tc_kernel<1>, gg, dim3(256), 0, STREAM(stream), gp)
                    : np <= 32 ? launch_pdl(tree_gates_tc_kernel<2>, gg, dim3(256), 0, STREAM(stream), gp)
                               : launch_pdl(tree_gates_tc_kernel<3>, gg, dim3(256), 0, STREAM(stream), gp);
    if (bad) return check_launch("tree_gates_tc_kernel");
    TreeRecurParams rp{pr, bi, bf, br, t_buf, doc,
                       BFM(rg_hist) + (size_t)b0 * max_len * L * H,
                       BF(v0) + (size_t)b0 * d, BFM(v_ring) + (size_t)b0 * S * d,
                       BFM(y) + (size_t)b0 * d, nb, max_len, L, H, hd, np, S};
    if ((nb <= 4 ? launch_tree_recur<kRecurRows>(rp, H, nb, STREAM(stream))
                : launch_tree_recur<1>(rp, H, nb, STREAM(stream))))
      return check_launch("tree_recur_kernel");
  }
  return DH_OK;
}

extern "C" int dh_decode_mixer_in_gates(const float* x, const void* norm_w, const void* w3, void* v0,
                                        void* a_out, void* b_hist, const int64_t* t_buf,
                                        int max_len, int batch, int d, const void* w_gates_t,
                                        int np, int L, int H, float* pre, const int* doc_hist,
                                        int* status, void* stream) {
  DH_REQUIRE(x && norm_w && w3 && v0 && a_out && b_hist && t_buf && w_gates_t && pre, DH_ERR_ARG,
             "dh_decode_mixer_in_gates: null pointer");
  DH_REQUIRE(batch >= 1 && batch <= 8 && d % 32 == 0 && d >= 32 && d <= 1024 && L >= 1 &&
                 L <= kGateMaxL && np % 16 == 0 && np >= 3 * H && 16 * L * np * 2 <= kBulkSlotBytes &&
                 max_len > 0,
             DH_ERR_SHAPE, "dh_decode_mixer_in_gates: unsupported sizes (batch %d, d %d, L %d, np %d)",
             batch, d, L, np);
  DH_REQUIRE(aligned16(x) && aligned16(w3) && aligned16(w_gates_t), DH_ERR_ARG,
             "dh_decode_mixer_in_gates: pointers must be 16-byte aligned");
  constexpr size_t kMaxSmem = 227 * 1024;
  const size_t fixed = bulk_xs_bytes(1, d) + (size_t)kTcWarps * 16 * 16 * 4 + 16 * 17 * 4 +
                       (size_t)8 * kGateMaxL * 16 * 4 + sizeof(BulkShared) + 16;
  const int nslots = (int)std::min<size_t>(kBulkMaxSlots, (kMaxSmem - fixed) / kBulkSlotBytes);
  const size_t smem = fixed + (size_t)nslots * kBulkSlotBytes;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(mixer_gates_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMaxSmem);
    configured_dev = dev;
  }
  MixerGatesParams p{x, BF(norm_w), BF(w3), BFM(v0), BFM(a_out), BFM(b_hist), t_buf, BF(w_gates_t),
                     pre, doc_hist, d, batch, max_len, L, np, 3 * H};
  const int grid = std::min(3 * d / 16, sm_count());
  // one 8-column mma tile of lockstep rows (up to 8 rows)
  if (launch_pdl(mixer_gates_kernel<1>, dim3(grid), dim3(kBulkThreads), smem, STREAM(stream), p, nslots,
                 status, wait_limit()))
    return check_launch("mixer_gates_kernel");
  return DH_OK;
}

extern "C" int dh_decode_tree_recur(const float* bi, const float* bf, const float* br,
                                    const int64_t* t_buf, float* pre, int np, void* rg_hist,
                                    const void* v0, void* v_ring, void* y, const int* doc_hist,
                                    int batch, int max_len, int L, int H, int hd, void* stream) {
  DH_REQUIRE(bi && bf && br && t_buf && pre && rg_hist && v0 && v_ring && y, DH_ERR_ARG,
             "dh_decode_tree_recur: null pointer");
  DH_REQUIRE(batch >= 1 && L >= 1 && L <= 16 && H >= 1 && hd >= 1 && hd <= 64 && np >= 3 * H,
             DH_ERR_SHAPE, "dh_decode_tree_recur: unsupported sizes (L=%d H=%d hd=%d np=%d)", L, H,
             hd, np);
  const int d = H * hd, S = (1 << (L + 1)) - 2;
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    TreeRecurParams rp{pre + (size_t)b0 * L * np, bi, bf, br, t_buf,
                       doc_hist ? doc_hist + (size_t)b0 * max_len : nullptr,
                       BFM(rg_hist) + (size_t)b0 * max_len * L * H,
                       BF(v0) + (size_t)b0 * d, BFM(v_ring) + (size_t)b0 * S * d,
                       BFM(y) + (size_t)b0 * d, nb, max_len, L, H, hd, np, S};
    if ((nb <= 4 ? launch_tree_recur<kRecurRows>(rp, H, nb, STREAM(stream))
                : launch_tree_recur<1>(rp, H, nb, STREAM(stream))))
      return check_launch("tree_recur_kernel");
  }
  return DH_OK;
}

extern "C" int dh_decode_linear_residual(const void* y, const void* w, float* x, float* x_copy,
                                         int batch, int k, int d_out, int* status, void* stream) {
  DH_REQUIRE(y && w && x, DH_ERR_ARG, "dh_decode_linear_residual: null pointer");
  DH_REQUIRE(d_out % 2 == 0, DH_ERR_SHAPE, "dh_decode_linear_residual: odd output width");
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    GemvIn in{BF(y) + (size_t)b0 * k, 0, nullptr, k, nb, status};
    EpiResidual e{BF(w), d_out, k, x + (size_t)b0 * d_out,
                  x_copy ? x_copy + (size_t)b0 * d_out : nullptr};
    const int rc = launch_gemv(in, e, d_out / 2, STREAM(stream));
    if (rc) return rc;
  }
  return DH_OK;
}

template <int MAXB>
int launch_ffn_bulk(const FfnParams& prm, int* status, cudaStream_t st) {
  constexpr size_t kMaxSmem = 227 * 1024;
  const size_t fixed = bulk_xs_bytes(MAXB > 8 ? 2 : 1, prm.d) + (size_t)kTcWarps * 16 * 16 * 4 +
                       16 * 17 * 4 + MAXB * 8 * 4 + sizeof(BulkShared) + 16;
  const int nslots = (int)std::min<size_t>(kBulkMaxSlots, (kMaxSmem - fixed) / kBulkSlotBytes);
  const size_t smem = fixed + (size_t)nslots * kBulkSlotBytes;
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(ffn_bulk_kernel<MAXB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)kMaxSmem);
    configured_dev = dev;
  }
  const int grid = std::min((prm.ff + 7) / 8, sm_count());
  if (launch_pdl(ffn_bulk_kernel<MAXB>, dim3(grid), dim3(kBulkThreads), smem, st, prm, nslots, status,
                 wait_limit()))
    return check_launch("ffn_bulk_kernel");
  return DH_OK;
}

extern "C" int dh_decode_ffn(const float* x_in, const void* norm_w, const void* w_gate,
                             const void* w_up, const void* w_down_t, float* x, int batch, int d,
                             int ff, int* status, void* stream) {
  DH_REQUIRE(x_in && norm_w && w_gate && w_up && w_down_t && x, DH_ERR_ARG,
             "dh_decode_ffn: null pointer");
  DH_REQUIRE(d % 8 == 0 && d <= 2048 && ff >= 1 && batch >= 1, DH_ERR_SHAPE,
             "dh_decode_ffn: unsupported sizes d=%d ff=%d", d, ff);
  DH_REQUIRE(aligned16(x_in) && aligned16(x) && aligned16(w_gate) && aligned16(w_up) &&
                 aligned16(w_down_t),
             DH_ERR_ARG, "dh_decode_ffn: pointers must be 16-byte aligned");
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(ffn_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, 2048 * 2);
    cudaFuncSetAttribute(ffn_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, 4 * 2048 * 2);
    cudaFuncSetAttribute(ffn_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         16 * 2048 * 2);
    configured_dev = dev;
  }
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    if (d <= 1024 && d % 32 == 0) {  // tensor cores, weights by bulk copies
      FfnParams prm{x_in + (size_t)b0 * d, BF(norm_w), BF(w_gate), BF(w_up), BF(w_down_t),
                    x + (size_t)b0 * d, d, ff, nb, 0};
      const int rc = nb == 1   ? launch_ffn_bulk<1>(prm, status, STREAM(stream))
                     : nb == 2 ? launch_ffn_bulk<2>(prm, status, STREAM(stream))
                     : nb <= 4 ? launch_ffn_bulk<4>(prm, status, STREAM(stream))
                     : nb <= 8 ? launch_ffn_bulk<8>(prm, status, STREAM(stream))
                               : launch_ffn_bulk<16>(prm, status, STREAM(stream));
      if (rc) return rc;
      continue;
    }
    const int maxb = nb == 1 ? 1 : (nb <= 4 ? 4 : 16);
    // one wave of CTAs at small batches; more u elements per CTA (fewer
    // atomic row updates) at large batches
    const int upc = maxb >= 16 ? kFfnMaxUpc
                               : std::min(kFfnMaxUpc, std::max(8, (ff + sm_count() - 1) / sm_count()));
    FfnParams prm{x_in + (size_t)b0 * d, BF(norm_w), BF(w_gate), BF(w_up), BF(w_down_t),
                  x + (size_t)b0 * d, d, ff, nb, upc};
    const dim3 grid((ff + upc - 1) / upc);
    const size_t smem = (size_t)maxb * d * 2;
    const int bad = maxb == 1 ? launch_pdl(ffn_kernel<1>, grid, dim3(kFfnWarps * 32), smem,
                                           STREAM(stream), prm)
                    : maxb == 4 ? launch_pdl(ffn_kernel<4>, grid, dim3(kFfnWarps * 32), smem,
                                             STREAM(stream), prm)
                                : launch_pdl(ffn_kernel<16>, grid, dim3(kFfnWarps * 32), smem,
                                             STREAM(stream), prm);
    if (bad) return check_launch("ffn_kernel");
  }
  return DH_OK;
}

extern "C" int dh_decode_ffn_in(const float* x, const void* norm_w, const void* w_gate,
                                const void* w_up, void* u, int batch, int d, int ff,
                                int* status, void* stream) {
  DH_REQUIRE(x && norm_w && w_gate && w_up && u, DH_ERR_ARG, "dh_decode_ffn_in: null pointer");
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    GemvIn in{x + (size_t)b0 * d, 1, BF(norm_w), d, nb, status};
    EpiSwiglu e{BF(w_gate), BF(w_up), ff, d, BFM(u) + (size_t)b0 * ff};
    int rc = launch_gemv(in, e, ff, STREAM(stream));
    if (rc) return rc;
  }
  return DH_OK;
}

extern "C" int dh_decode_attn_in(const float* x, const void* norm_w, const void* wqkv,
                                 const float* rope_cos, const float* rope_sin, void* q,
                                 void* k_cache, void* v_cache, const int64_t* t_buf, int max_len,
                                 int batch, int d, int H, int* status, void* stream) {
  DH_REQUIRE(x && norm_w && wqkv && rope_cos && rope_sin && q && k_cache && v_cache && t_buf,
             DH_ERR_ARG, "dh_decode_attn_in: null pointer");
  DH_REQUIRE(H > 0 && d % H == 0 && (d / H) % 2 == 0, DH_ERR_SHAPE, "dh_decode_attn_in: bad heads");
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    GemvIn in{x + (size_t)b0 * d, 1, BF(norm_w), d, nb, status};
    EpiQkvRope e{BF(wqkv), d, d, d / H, max_len, rope_cos, rope_sin,
                 BFM(q) + (size_t)b0 * d, BFM(k_cache) + (size_t)b0 * max_len * d,
                 BFM(v_cache) + (size_t)b0 * max_len * d, t_buf};
    int rc = launch_gemv(in, e, 3 * d / 2, STREAM(stream));
    if (rc) return rc;
  }
  return DH_OK;
}

extern "C" int dh_decode_attn(const void* q, const void* k_cache, const void* v_cache, void* y,
                              const int64_t* t_buf, float* part, int* counters, int nsplit,
                              int batch, int max_len, int H, int hd, int window, void* stream) {
  DH_REQUIRE(q && k_cache && v_cache && y && t_buf, DH_ERR_ARG, "dh_decode_attn: null pointer");
  DH_REQUIRE(hd == 64, DH_ERR_SHAPE, "dh_decode_attn: head_dim %d unsupported (64 only)", hd);
  DH_REQUIRE(nsplit >= 1 && nsplit <= 64, DH_ERR_SHAPE, "dh_decode_attn: nsplit %d", nsplit);
  DH_REQUIRE(nsplit == 1 || (part && counters), DH_ERR_ARG,
             "dh_decode_attn: nsplit > 1 needs part and counters scratch");
  const int span = (window > 0 && window < max_len) ? window : max_len;
  const int cap = (span + nsplit - 1) / nsplit;
  DH_REQUIRE(cap <= 12288, DH_ERR_SHAPE, "dh_decode_attn: window chunk %d too large", cap);
  const size_t smem = (size_t)cap * sizeof(float);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         12288 * 4);
    configured_dev = dev;
  }
  const int d = H * hd;
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    AttnParams p{BF(q) + (size_t)b0 * d, BF(k_cache) + (size_t)b0 * max_len * d,
                 BF(v_cache) + (size_t)b0 * max_len * d, BFM(y) + (size_t)b0 * d, t_buf,
                 part ? part + (size_t)b0 * H * nsplit * (hd + 2) : nullptr,
                 counters ? counters + (size_t)b0 * H : nullptr, max_len, H, window, cap};
    if (launch_pdl(attn_decode_kernel, dim3(H, nb, nsplit), dim3(128), smem, STREAM(stream), p))
      return check_launch("attn_decode_kernel");
  }
  return DH_OK;
}

extern "C" int dh_decode_logits(const float* x, const void* norm_w, const void* emb, void* logits,
                                int batch, int d, int vocab, int* status, void* stream) {
  DH_REQUIRE(x && norm_w && emb && logits, DH_ERR_ARG, "dh_decode_logits: null pointer");
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    GemvIn in{x + (size_t)b0 * d, 1, BF(norm_w), d, nb, status};
    EpiLogits e{BF(emb), vocab, d, BFM(logits) + (size_t)b0 * vocab};
    int rc = launch_gemv(in, e, (vocab + 1) / 2, STREAM(stream));
    if (rc) return rc;
  }
  return DH_OK;
}

extern "C" int dh_decode_doc_step(const int64_t* tokens, const int64_t* t_buf, int* doc_hist,
                                  int64_t* last_tok, int64_t eot, int batch, int max_len,
                                  void* stream) {
  DH_REQUIRE(tokens && t_buf && doc_hist && last_tok, DH_ERR_ARG,
             "dh_decode_doc_step: null pointer");
  DH_REQUIRE(batch >= 1 && max_len >= 1, DH_ERR_SHAPE, "dh_decode_doc_step: bad sizes");
  if (launch_pdl(doc_step_kernel, dim3((batch + 127) / 128), dim3(128), 0, STREAM(stream), tokens,
                 t_buf, doc_hist, last_tok, eot, max_len, batch))
    return check_launch("doc_step_kernel");
  return DH_OK;
}

extern "C" int dh_decode_argmax(const void* logits, int64_t* next_tokens, int64_t* out, int batch,
                                int vocab, void* stream) {
  DH_REQUIRE(logits && next_tokens, DH_ERR_ARG, "dh_decode_argmax: null pointer");
  DH_REQUIRE(batch >= 1 && vocab >= 1, DH_ERR_SHAPE, "dh_decode_argmax: bad sizes");
  if (launch_pdl(argmax_kernel, dim3(batch), dim3(1024), 0, STREAM(stream), BF(logits), vocab,
                 next_tokens, out))
    return check_launch("argmax_kernel");
  return DH_OK;
}

extern "C" int dh_decode_sample_top_k(const void* logits, int64_t* next_tokens, int64_t* out,
                                      int batch, int vocab, int top_k, float temperature,
                                      unsigned long long seed, const int64_t* t_buf, void* stream) {
  DH_REQUIRE(logits && next_tokens && t_buf, DH_ERR_ARG, "dh_decode_sample_top_k: null pointer");
  DH_REQUIRE(batch >= 1 && vocab >= 1 && top_k >= 1, DH_ERR_SHAPE,
             "dh_decode_sample_top_k: bad sizes");
  const float inv_t = 1.0f / (temperature > 1e-6f ? temperature : 1e-6f);
  if (launch_pdl(sample_top_k_kernel, dim3(batch), dim3(1024), 0, STREAM(stream), BF(logits), vocab,
                 top_k, inv_t, seed, t_buf, next_tokens, out))
    return check_launch("sample_top_k_kernel");
  return DH_OK;
}

extern "C" int dh_decode_advance(int64_t* t_buf, void* stream) {
  DH_REQUIRE(t_buf, DH_ERR_ARG, "dh_decode_advance: null pointer");
  if (launch_pdl(advance_kernel, dim3(1), dim3(1), 0, STREAM(stream), t_buf))
    return check_launch("advance_kernel");
  return DH_OK;
}

// ------------------------------------------- split-window attention, no allocation
// dh_decode_attn_noalloc runs the same split-window kernel as dh_decode_attn,
// but its two scratch buffers live in this file's own device storage instead
// of memory the caller passes in.  It exists for callers that cannot allocate
// device memory: a host that binds the C ABI from another language runtime
// and owns no CUDA allocator, or a serving loop that must not call cudaMalloc
// between steps (it can synchronise the whole device, and it can fail when
// the pool is nearly full, in the middle of a decode step).
//
// Limits: batch * H * nsplit * (hd + 2) <= kNoAllocPartFloats (131072 floats,
// 512 KiB) and batch * H <= kNoAllocCounters (1024).  Larger requests are
// rejected with DH_ERR_SHAPE before anything is launched.
//
// What must start at zero: the counters.  They are zeroed once, when a device
// is set up, and every call leaves them zero again (the last CTA of each
// (row, head) resets its own counter).  The partial results need no initial
// value: each split writes its slot before the combining CTA reads it.
//
// The first call on each device does the setup (symbol lookup, kernel
// attribute, zeroing of the counters, all on that device while it is
// current); make that first call before any stream capture.  There is one
// scratch area per device: calls whose executions overlap in time on the same
// device (two streams, two host threads) race on it and must be serialised by
// the caller.
namespace dh {

constexpr int kNoAllocPartFloats = 131072;
constexpr int kNoAllocCounters = 1024;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) float g_noalloc_part[kNoAllocPartFloats];
static __device__ __align__(256) int g_noalloc_counters[kNoAllocCounters];

struct NoAllocScratch {
  float* part;
  int* counters;
};

static NoAllocScratch g_noalloc_dev[kNoAllocMaxDevices];  // zero until set up
static std::mutex g_noalloc_mu;

static int noalloc_scratch(cudaStream_t st, NoAllocScratch* out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(DH_ERR_CUDA, "dh_decode_attn_noalloc: cudaGetDevice: %s",
                                         cudaGetErrorString(e));
  if (dev < 0 || dev >= kNoAllocMaxDevices)
    return set_error(DH_ERR_DEVICE, "dh_decode_attn_noalloc: device %d beyond %d", dev,
                     kNoAllocMaxDevices);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  NoAllocScratch& s = g_noalloc_dev[dev];
  if (!s.part) {
    void* part = nullptr;
    void* counters = nullptr;
    e = cudaGetSymbolAddress(&part, g_noalloc_part);
    if (e != cudaSuccess)
      return set_error(DH_ERR_CUDA, "dh_decode_attn_noalloc: scratch symbol lookup: %s",
                       cudaGetErrorString(e));
    e = cudaGetSymbolAddress(&counters, g_noalloc_counters);
    if (e != cudaSuccess)
      return set_error(DH_ERR_CUDA, "dh_decode_attn_noalloc: counter symbol lookup: %s",
                       cudaGetErrorString(e));
    e = cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             12288 * 4);
    if (e != cudaSuccess)
      return set_error(DH_ERR_CUDA, "dh_decode_attn_noalloc: kernel attribute: %s",
                       cudaGetErrorString(e));
    e = cudaMemsetAsync(counters, 0, sizeof(int) * kNoAllocCounters, st);
    if (e != cudaSuccess)
      return set_error(DH_ERR_CUDA, "dh_decode_attn_noalloc: zeroing counters: %s",
                       cudaGetErrorString(e));
    s.part = static_cast<float*>(part);
    s.counters = static_cast<int*>(counters);
  }
  *out = s;
  return DH_OK;
}

}  // namespace dh

extern "C" int dh_decode_attn_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                      void* y, const int64_t* t_buf, int nsplit, int batch,
                                      int max_len, int H, int hd, int window, void* stream) {
  DH_REQUIRE(q && k_cache && v_cache && y && t_buf, DH_ERR_ARG,
             "dh_decode_attn_noalloc: null pointer");
  DH_REQUIRE(hd == 64, DH_ERR_SHAPE, "dh_decode_attn_noalloc: head_dim %d unsupported (64 only)",
             hd);
  DH_REQUIRE(nsplit >= 1 && nsplit <= 64, DH_ERR_SHAPE, "dh_decode_attn_noalloc: nsplit %d",
             nsplit);
  DH_REQUIRE(batch >= 1 && H >= 1 && max_len >= 1, DH_ERR_SHAPE,
             "dh_decode_attn_noalloc: batch %d, H %d, max_len %d", batch, H, max_len);
  const long long part_floats = (long long)batch * H * nsplit * (hd + 2);
  DH_REQUIRE(part_floats <= kNoAllocPartFloats, DH_ERR_SHAPE,
             "dh_decode_attn_noalloc: batch*H*nsplit*(hd+2) = %lld floats of partial results "
             "exceeds the built-in scratch of %d floats",
             part_floats, kNoAllocPartFloats);
  DH_REQUIRE((long long)batch * H <= kNoAllocCounters, DH_ERR_SHAPE,
             "dh_decode_attn_noalloc: batch*H = %lld exceeds the built-in %d counters",
             (long long)batch * H, kNoAllocCounters);
  const int span = (window > 0 && window < max_len) ? window : max_len;
  const int cap = (span + nsplit - 1) / nsplit;
  DH_REQUIRE(cap <= 12288, DH_ERR_SHAPE, "dh_decode_attn_noalloc: window chunk %d too large", cap);
  NoAllocScratch s;
  const int rc = noalloc_scratch(STREAM(stream), &s);
  if (rc) return rc;
  const size_t smem = (size_t)cap * sizeof(float);
  const int d = H * hd;
  for (int b0 = 0; b0 < batch; b0 += kMaxRows) {
    const int nb = batch - b0 < kMaxRows ? batch - b0 : kMaxRows;
    AttnParams p{BF(q) + (size_t)b0 * d, BF(k_cache) + (size_t)b0 * max_len * d,
                 BF(v_cache) + (size_t)b0 * max_len * d, BFM(y) + (size_t)b0 * d, t_buf,
                 s.part + (size_t)b0 * H * nsplit * (hd + 2), s.counters + (size_t)b0 * H,
                 max_len, H, window, cap};
    if (launch_pdl(attn_decode_kernel, dim3(H, nb, nsplit), dim3(128), smem, STREAM(stream), p))
      return check_launch("attn_decode_kernel");
  }
  return DH_OK;
}

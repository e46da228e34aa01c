// Sliding-window causal attention for the parallel forward
// (modeling_dispatcher.py:168-185: keys s with t - window < s <= t, scale
// 1/sqrt(hd); plain causal when the window covers the sequence).
//
// Flash-style single pass: a CTA owns 64 query rows of one (sequence, head);
// each of its 4 warps holds 16 rows of Q as tensor-core fragments and walks
// only the key blocks that intersect the window, keeping an online softmax in
// registers.  K/V blocks of 64 keys are double-buffered in shared memory with
// cp.async; S = Q K^T and O += P V use mma.sync m16n8k16 (bf16 in, fp32 acc).
// q and k arrive already rotated (RoPE applied by dh_rope_qk).
#include <math.h>

#include "common.cuh"

namespace dh {
namespace {

constexpr int HD = 64;
constexpr int BQ = 64;
constexpr int BKV = 64;
constexpr int PITCH = HD + 8;  // bf16 elements per smem row (144 B): conflict-free ldmatrix

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)), "l"(gmem),
               "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct AttnArgs {
  const __nv_bfloat16* qkv;  // (B*T, ld): q at [0,d), k at [d,2d), v at [2d,3d)
  int ld;
  __nv_bfloat16* out;
  int ldo;
  int T, H, window;
};

// load 64 rows x 64 bf16 of one head into a padded smem tile (128 threads)
__device__ __forceinline__ void load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int ld,
                                          int row0, int nrows_valid) {
  const int tid = threadIdx.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = tid + i * 128;  // 512 chunks of 16 B
    const int r = c >> 3, part = c & 7;
    const bool ok = r < nrows_valid;
    const __nv_bfloat16* g = src + (size_t)(ok ? row0 + r : 0) * ld + part * 8;
    cp_async16(dst + r * PITCH + part * 8, g, ok);
  }
}

__global__ void __launch_bounds__(128) attn_prefill_kernel(AttnArgs a) {
  __shared__ __align__(128) __nv_bfloat16 sQ[BQ * PITCH];
  __shared__ __align__(128) __nv_bfloat16 sK[2][BKV * PITCH];
  __shared__ __align__(128) __nv_bfloat16 sV[2][BKV * PITCH];
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = a.T, d = a.H * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q0 = qb * BQ;
  const bool windowed = a.window > 0 && a.window < T;
  const int W = windowed ? a.window : T + 1;
  const __nv_bfloat16* base = a.qkv + (size_t)b * T * a.ld;
  const __nv_bfloat16* qg = base + h * HD;
  const __nv_bfloat16* kg = base + d + h * HD;
  const __nv_bfloat16* vg = base + 2 * d + h * HD;

  int kstart = q0 - W + 1;
  if (kstart < 0) kstart = 0;
  kstart = (kstart / BKV) * BKV;
  int kend = q0 + BQ;
  if (kend > T) kend = T;
  const int nblk = (kend - kstart + BKV - 1) / BKV;

  load_tile(sQ, qg, a.ld, q0, T - q0);
  load_tile(sK[0], kg, a.ld, kstart, T - kstart);
  load_tile(sV[0], vg, a.ld, kstart, T - kstart);
  cp_async_commit();

  // per-warp state: 16 query rows; this thread owns rows g and g+8
  const int g = lane >> 2, tq = lane & 3;
  const int qrow0 = q0 + warp * 16 + g, qrow1 = qrow0 + 8;
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
  uint32_t qf[4][4];

  for (int it = 0; it < nblk; ++it) {
    const int buf = it & 1;
    const int k0 = kstart + it * BKV;
    if (it + 1 < nblk) {
      load_tile(sK[buf ^ 1], kg, a.ld, k0 + BKV, T - (k0 + BKV));
      load_tile(sV[buf ^ 1], vg, a.ld, k0 + BKV, T - (k0 + BKV));
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (it == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const int mi = lane >> 3;
        const int row = warp * 16 + (lane & 7) + (mi & 1) * 8;
        const int col = kk * 16 + (mi >> 1) * 8;
        ldsm_x4(qf[kk], sQ + row * PITCH + col);
      }
    }
    // S = Q K^T for 64 keys: 8 n-tiles of 8 keys
    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of n-tiles
        uint32_t kf[4];
        const int mi = lane >> 3;
        const int key = np * 16 + (lane & 7) + (mi >> 1) * 8;
        const int col = kk * 16 + (mi & 1) * 8;
        ldsm_x4(kf, sK[buf] + key * PITCH + col);
        mma16816(s[2 * np], qf[kk], kf[0], kf[1]);
        mma16816(s[2 * np + 1], qf[kk], kf[2], kf[3]);
      }
    }
    // mask + online softmax (base-2)
    float bm0 = -INFINITY, bm1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + nt * 8 + tq * 2 + (e & 1);
        const int qr = e < 2 ? qrow0 : qrow1;
        const bool valid = key < T && key <= qr && qr - key < W;
        const float v = valid ? s[nt][e] * sl2 : -INFINITY;
        s[nt][e] = v;
        if (e < 2) bm0 = fmaxf(bm0, v); else bm1 = fmaxf(bm1, v);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      bm0 = fmaxf(bm0, __shfl_xor_sync(0xffffffffu, bm0, off));
      bm1 = fmaxf(bm1, __shfl_xor_sync(0xffffffffu, bm1, off));
    }
    const float mn0 = fmaxf(m0, bm0), mn1 = fmaxf(m1, bm1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0, base1 = mn1 == -INFINITY ? 0.f : mn1;
    const float c0 = exp2f(m0 - base0), c1 = exp2f(m1 - base1);
    m0 = mn0;
    m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      s[nt][0] = exp2f(s[nt][0] - base0);
      s[nt][1] = exp2f(s[nt][1] - base0);
      s[nt][2] = exp2f(s[nt][2] - base1);
      s[nt][3] = exp2f(s[nt][3] - base1);
      rs0 += s[nt][0] + s[nt][1];
      rs1 += s[nt][2] + s[nt][3];
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
      o[nt][0] *= c0;
      o[nt][1] *= c0;
      o[nt][2] *= c1;
      o[nt][3] *= c1;
    }
    // O += P V: 4 key steps of 16, 8 dim tiles of 8
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {  // pairs of dim tiles
        uint32_t vf[4];
        const int mi = lane >> 3;
        const int key = kk * 16 + (lane & 7) + (mi & 1) * 8;
        const int col = dp * 16 + (mi >> 1) * 8;
        ldsm_x4_t(vf, sV[buf] + key * PITCH + col);
        mma16816(o[2 * dp], pa, vf[0], vf[1]);
        mma16816(o[2 * dp + 1], pa, vf[2], vf[3]);
      }
    }
    __syncthreads();  // buffer `buf` is refilled by the next iteration's prefetch
  }
  // row sums are partial per thread quad: reduce
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, off);
    l1 += __shfl_xor_sync(0xffffffffu, l1, off);
  }
  const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  __nv_bfloat16* ob = a.out + (size_t)b * T * a.ldo + h * HD;
#pragma unroll
  for (int nt = 0; nt < 8; ++nt) {
    const int col = nt * 8 + tq * 2;
    if (qrow0 < T)
      *reinterpret_cast<uint32_t*>(ob + (size_t)qrow0 * a.ldo + col) =
          pack2(o[nt][0] * inv0, o[nt][1] * inv0);
    if (qrow1 < T)
      *reinterpret_cast<uint32_t*>(ob + (size_t)qrow1 * a.ldo + col) =
          pack2(o[nt][2] * inv1, o[nt][3] * inv1);
  }
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" int dh_window_attn_prefill(const void* qkv, int ld, void* out, int ldo, int batch,
                                      int T, int H, int hd, int window, void* stream) {
  DH_REQUIRE(qkv && out, DH_ERR_ARG, "dh_window_attn_prefill: null pointer");
  DH_REQUIRE(hd == HD, DH_ERR_SHAPE, "dh_window_attn_prefill: head_dim %d (64 only)", hd);
  DH_REQUIRE(ld % 8 == 0 && ldo % 2 == 0 && T > 0 && batch > 0, DH_ERR_SHAPE,
             "dh_window_attn_prefill: bad sizes");
  AttnArgs a{reinterpret_cast<const __nv_bfloat16*>(qkv), ld,
             reinterpret_cast<__nv_bfloat16*>(out), ldo, T, H, window};
  dim3 grid((T + BQ - 1) / BQ, H, batch);
  attn_prefill_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
  return check_launch("attn_prefill_kernel");
}

// bf16 GEMM on the 5th-generation tensor cores: c[m,n] = a[m,k]·w[n,k]ᵀ (+ c), fp32 accumulate.
//
// The step's projections are weight-streaming GEMMs: m = batch·(k+1) ≤ 256 token rows against
// n·k weights read once from HBM. The weight tile is therefore the MMA "A" operand
// (M_mma = 128 weight rows = 128 output columns) and the token rows are the "B" operand
// (N_mma = MT ≤ 256), so one CTA holds D[128 × MT] fp32 in TMEM and streams its weight rows
// once. Warp roles (192 threads): warp 0 issues TMA loads into a STAGES-deep ring of
// 128B-swizzled tiles, warp 1 owns TMEM and issues tcgen05.mma (one thread), warps 2-5 drain
// TMEM with tcgen05.ld and write bf16. When n/128 tiles cannot fill the SMs, the K range is
// split; every split writes an fp32 partial and a second, fully parallel kernel sums the
// partials in split order (results do not depend on CTA scheduling).
//
// Every mbarrier wait is bounded; a wait that runs out records an error code in a device
// flag (read by qsp_device_status) and the CTA finishes without hanging the GPU.
#include "qsp_common.cuh"
#include "qsp_tc.cuh"

#include <cuda.h>
#include <stdlib.h>

#include <mutex>
#include <unordered_map>

namespace qsp {

__device__ int g_qsp_dev_error = 0;

constexpr int TC_MM = 128;          // MMA M (weight rows per accumulator)
constexpr int TC_BK = 64;           // K elements per stage (128 bytes of bf16: one swizzle row)
constexpr int TC_THREADS = 192;
constexpr uint32_t WAIT_LIMIT = 1u << 24;

// ------------------------------------------------------------------ PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false (and the device error flag set to `code`) if the phase never completes.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int code) {
  for (uint32_t i = 0; i < WAIT_LIMIT; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 256) __nanosleep(64);
  }
  atomicExch(&g_qsp_dev_error, code);
  return false;
}
// mbar_wait by all lanes of a converged warp (same result in every lane)
__device__ __forceinline__ bool mbar_wait_w(uint64_t* bar, uint32_t parity, int code) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, code));
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
// Weight tiles are read once per launch: load them with an L2 evict-first policy so that they
// do not displace the activations, split-K partials and state that the step re-reads.
__device__ __forceinline__ void tma_load_2d_evict_first(void* dst, const CUtensorMap* map, uint64_t* bar, int x,
                                                        int y) {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], "
      "[%2], %5;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(pol)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand tile written by TMA with 128-byte swizzling: rows of 128 B, 8-row groups
// 1024 B apart (stride byte offset), descriptor version 1, layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// kind::f16 instruction descriptor: D fp32, A and B bf16, both K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// BN weight rows per work unit: 128 (one accumulator) or 256 (two M=128 MMAs share each
// activation tile, halving the activation re-reads of a wide projection). KPS k-blocks per ring
// stage: with KPS = 2 each operand of a stage arrives as ONE 3-D TMA box spanning two k-blocks
// ([k-block][rows][128 B] in shared memory). A TMA unit moves a bounded number of boxes per
// microsecond (about 3.4 per SM on B200, whatever their size up to 32 KB), so small boxes —
// 16 KB weight tiles, 4–8 KB activation tiles of few token rows — cap an SM's ingest well
// below its ~110 GB/s port; two k-blocks per box double the bytes per box.
template <int MT, int BN, int KPS = 1>
struct TcCfg {
  static constexpr int TC_BN = BN;
  static constexpr int W_BYTES = KPS * BN * TC_BK * 2;
  static constexpr int NACC = BN / TC_MM;   // accumulators per unit
  static constexpr int X_BYTES = KPS * MT * TC_BK * 2;
  static constexpr int STAGE_BYTES = W_BYTES + X_BYTES;
  // one persistent CTA per SM: the ring fills ~192 KB of shared memory
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  // NACC accumulators of MT fp32 columns per unit; double-buffered (the epilogue of one unit
  // overlaps the MMAs of the next) when two sets fit in the 512 TMEM columns
  static constexpr int ACC_COLS = MT < 32 ? 32 : MT;
  static constexpr int UNIT_COLS = NACC * ACC_COLS;
  static constexpr int ACC_BUFS = (2 * UNIT_COLS <= 512) ? 2 : 1;
  static constexpr int TMEM_COLS = ACC_BUFS * UNIT_COLS;
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024 + 256;
};

struct TcArgs {
  __nv_bfloat16* c;
  int64_t ldc;
  int m, n, n_kb, kb_per_split, splits, accumulate;
  int m_tiles, n_tiles, units;   // work unit u: split u / tiles, tile u % tiles (m-tile fastest)
  float* partial;  // [splits][m_tiles*MT][n_tiles*BN]
  // K-split tail (unsplit plans only): units from full_units on cover tiles full_units.. in
  // tail_split K slices of tail_kps k-blocks each, written as fp32 partials
  // [tail_split][MT][(tiles − full_units)·BN] and summed by a merge
  int full_units, tail_split, tail_kps;
};

struct TcUnit {
  int tile, slice, kb0, nk;
  bool tail;
};
__device__ __forceinline__ TcUnit tc_unit(const TcArgs& A, int u, int tiles) {
  TcUnit r;
  if (A.tail_split > 0 && u >= A.full_units) {
    const int v = u - A.full_units;
    r.tile = A.full_units + v / A.tail_split;
    r.slice = v % A.tail_split;
    r.kb0 = r.slice * A.tail_kps;
    r.nk = min(A.n_kb, r.kb0 + A.tail_kps) - r.kb0;
    r.tail = true;
  } else {
    r.slice = u / tiles;
    r.tile = u % tiles;
    r.kb0 = r.slice * A.kb_per_split;
    r.nk = min(A.n_kb, r.kb0 + A.kb_per_split) - r.kb0;
    r.tail = false;
  }
  return r;
}

// What happens to the product after the split-K merge (the unsplit kernel always stores c).
struct GemmEpi {
  int kind;                     // GEMM_EPI_STORE / _RESNORM / _SWIGLU
  const __nv_bfloat16* norm_w;  // RESNORM: RMSNorm weight (1+w convention)
  __nv_bfloat16* y;             // RESNORM: normed output; SWIGLU: activation output
  int64_t ldy;
  float eps;
};
enum { GEMM_EPI_STORE = 0, GEMM_EPI_RESNORM = 1, GEMM_EPI_SWIGLU = 2 };

// ---------------------------------------------------------------- split-K merges
// Partials are summed in split order (deterministic); loads are issued four splits at a time.
__device__ __forceinline__ float4 merge4(const float* __restrict__ p, int splits, int64_t stride) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < splits; s += 4) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      v[u] = (s + u < splits) ? __ldcg(reinterpret_cast<const float4*>(p + (s + u) * stride)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (s + u < splits) {
        acc.x += v[u].x; acc.y += v[u].y; acc.z += v[u].z; acc.w += v[u].w;
      }
    }
  }
  return acc;
}

// The same sum (same order) with up to eight splits' loads in flight at once.
__device__ __forceinline__ float4 merge8(const float* __restrict__ p, int splits, int64_t stride) {
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int s = 0; s < splits; s += 8) {
    float4 v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u)
      v[u] = (s + u < splits) ? __ldcg(reinterpret_cast<const float4*>(p + (s + u) * stride)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      if (s + u < splits) {
        acc.x += v[u].x; acc.y += v[u].y; acc.z += v[u].z; acc.w += v[u].w;
      }
    }
  }
  return acc;
}

// c = round(Σ partial) (+ c)
__global__ void __launch_bounds__(256) splitk_store_kernel(const float* __restrict__ partial, int splits,
                                                           int64_t split_stride, int ldp,
                                                           __nv_bfloat16* __restrict__ c, int64_t ldc, int n,
                                                           int accumulate) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.y;
  const int col = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (col >= n) return;
  const float4 acc = merge4(partial + (int64_t)row * ldp + col, splits, split_stride);
  const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
  __nv_bfloat16* o = c + (int64_t)row * ldc + col;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    if (col + j >= n) break;
    float r = dt<__nv_bfloat16>::round(a4[j]);
    if (accumulate) r += __bfloat162float(o[j]);
    o[j] = __float2bfloat16_rn(r);
  }
}

// Residual add + the following RMSNorm, one CTA per row:
// x := round(x + round(Σ partial)); y = round(x̂·(1 + w)) with x̂ = x·rsqrt(mean(x²) + eps).
// One CTA of 512 threads per row: a 2048-column row is one float4 per thread, so every split
// of it is in flight at once (the row's latency is one L2 round trip, not one per four splits).
constexpr int RN_THREADS = 512;
constexpr int RN_MAXV = 4;   // up to 8192 columns (512 threads x 4 x 4)
__global__ void __launch_bounds__(RN_THREADS) splitk_residual_rmsnorm_kernel(
    const float* __restrict__ partial, int splits, int64_t split_stride, int ldp, __nv_bfloat16* __restrict__ x,
    int64_t ldx, const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y, int64_t ldy, int n, float eps) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int row = blockIdx.x;
  float r[RN_MAXV][4];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < RN_MAXV; ++v) {
    const int col = (threadIdx.x + v * RN_THREADS) * 4;
    if (col < n) {
      const float4 acc = merge8(partial + (int64_t)row * ldp + col, splits, split_stride);
      const float a4[4] = {acc.x, acc.y, acc.z, acc.w};
      __nv_bfloat16* xo = x + (int64_t)row * ldx + col;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float val = dt<__nv_bfloat16>::round(dt<__nv_bfloat16>::round(a4[j]) + __bfloat162float(xo[j]));
        xo[j] = __float2bfloat16_rn(val);
        r[v][j] = val;
        ss = fmaf(val, val, ss);
      }
    }
  }
  const float tot = block_sum(ss, red);
  const float inv = rsqrtf(tot / (float)n + eps);
#pragma unroll
  for (int v = 0; v < RN_MAXV; ++v) {
    const int col = (threadIdx.x + v * RN_THREADS) * 4;
    if (col < n) {
      __nv_bfloat16* yo = y + (int64_t)row * ldy + col;
#pragma unroll
      for (int j = 0; j < 4; ++j) yo[j] = __float2bfloat16_rn(r[v][j] * inv * (__bfloat162float(w[col + j]) + 1.0f));
    }
  }
}

// SwiGLU of a fused [gate | up] projection: act = round(round(silu(round(g))) · round(u)).
__global__ void __launch_bounds__(256) splitk_swiglu_kernel(const float* __restrict__ partial, int splits,
                                                            int64_t split_stride, int ldp,
                                                            __nv_bfloat16* __restrict__ act, int64_t ld_act,
                                                            int inter) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.y;
  const int j = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (j >= inter) return;
  const float* p = partial + (int64_t)row * ldp;
  const float4 g = merge4(p + j, splits, split_stride);
  const float4 u = merge4(p + inter + j, splits, split_stride);
  const float g4[4] = {g.x, g.y, g.z, g.w}, u4[4] = {u.x, u.y, u.z, u.w};
  __nv_bfloat16* o = act + (int64_t)row * ld_act + j;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float s = dt<__nv_bfloat16>::round(siluf_(dt<__nv_bfloat16>::round(g4[q])));
    o[q] = __float2bfloat16_rn(s * dt<__nv_bfloat16>::round(u4[q]));
  }
}

// Operand loads of one ring stage: k-blocks kb .. kb+KPS-1 of rows [row, row + box rows).
// KPS = 1: a 2-D box at (kb·64, row); KPS = 2: a 3-D box at (0, row, kb) over the view
// [k-blocks][rows][64 elements] of the same row-major matrix (K a multiple of 64).
template <int KPS>
__device__ __forceinline__ void tc_load_w(void* dst, const CUtensorMap* map, uint64_t* bar, int kb, int row) {
  if (KPS == 1) {
    tc::tma_load_2d_evict_first_warp(dst, map, bar, kb * TC_BK, row);
  } else {
    asm volatile(
        "{\n\t.reg .pred e;\n\t.reg .b64 pol;\n\telect.sync _|e, 0xffffffff;\n\t"
        "createpolicy.fractional.L2::evict_first.b64 pol, 1.0;\n\t"
        "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4, "
        "%5}], [%2], pol;\n\t}" ::"r"(smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(0), "r"(row), "r"(kb)
        : "memory");
  }
}
template <int KPS>
__device__ __forceinline__ void tc_load_x(void* dst, const CUtensorMap* map, uint64_t* bar, int kb, int row) {
  if (KPS == 1) {
    tc::tma_load_2d_warp(dst, map, bar, kb * TC_BK, row);
  } else {
    asm volatile(
        "{\n\t.reg .pred e;\n\telect.sync _|e, 0xffffffff;\n\t"
        "@e cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];\n\t}" ::"r"(
            smem_u32(dst)),
        "l"(map), "r"(smem_u32(bar)), "r"(0), "r"(row), "r"(kb)
        : "memory");
  }
}

template <int MT, int BN, int KPS>
__global__ void __launch_bounds__(TC_THREADS, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, const TcArgs A) {
  using C = TcCfg<MT, BN, KPS>;
  constexpr int TC_BN = BN;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::STAGES * C::STAGE_BYTES);
  uint64_t* empty = full + C::STAGES;
  uint64_t* acc_full = empty + C::STAGES;   // [2]
  uint64_t* acc_empty = acc_full + 2;       // [2]
  uint32_t* tslot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = A.m_tiles * A.n_tiles;
  pdl_trigger();

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;

  if (warp == 0) {
    // TMA producer: one continuous ring across every k-block of every unit of this CTA. The
    // whole warp runs the loop; one elected lane issues (tcgen05/TMA issue from a lone lane of
    // a diverged warp is several times slower).
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_w) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_x) : "memory");
    }
    __syncwarp();
    // The weights do not depend on the previous kernel: the first ring pass issues its
    // weight tiles before the dependency wait, and its activation tiles after it.
    // a unit's k-blocks go in steps of KPS; step i covers k-blocks kb0 + KPS·((i + rot) % ns)
    int pre_kb[C::STAGES], pre_mb[C::STAGES];
    uint32_t npre = 0;
    for (int u = blockIdx.x; u < A.units && npre < (uint32_t)C::STAGES; u += gridDim.x) {
      const TcUnit U = tc_unit(A, u, tiles);
      const int mb = U.tile % A.m_tiles, nb = U.tile / A.m_tiles, kb0 = U.kb0;
      const int ns = (U.nk + KPS - 1) / KPS;
      const int rot = u % ns;
      for (int i = 0; i < ns && npre < (uint32_t)C::STAGES; ++i, ++npre) {
        const int kb = kb0 + KPS * ((i + rot) % ns);
        tc::mbar_expect_tx_warp(&full[npre], C::STAGE_BYTES);
        tc_load_w<KPS>(smem + npre * C::STAGE_BYTES, &tm_w, &full[npre], kb, nb * TC_BN);
        pre_kb[npre] = kb;
        pre_mb[npre] = mb;
      }
    }
    pdl_wait();
    for (uint32_t j = 0; j < npre; ++j)
      tc_load_x<KPS>(smem + j * C::STAGE_BYTES + C::W_BYTES, &tm_x, &full[j], pre_kb[j], pre_mb[j] * MT);
    uint32_t it = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < A.units && ok; u += gridDim.x) {
      const TcUnit U = tc_unit(A, u, tiles);
      const int mb = U.tile % A.m_tiles, nb = U.tile / A.m_tiles, kb0 = U.kb0;
      // units walk their k-blocks from a rotated start so concurrent CTAs read different
      // activation slabs
      const int ns = (U.nk + KPS - 1) / KPS;
      const int rot = u % ns;
      for (int i = 0; i < ns; ++i, ++it) {
        if (it < npre) continue;   // issued above
        const int kb = kb0 + KPS * ((i + rot) % ns);
        const int s = it % C::STAGES;
        const uint32_t ph = (it / C::STAGES) & 1u;
        if (it >= (uint32_t)C::STAGES && !mbar_wait_w(&empty[s], ph ^ 1u, 101)) { ok = false; break; }
        uint8_t* st = smem + s * C::STAGE_BYTES;
        tc::mbar_expect_tx_warp(&full[s], C::STAGE_BYTES);
        tc_load_w<KPS>(st, &tm_w, &full[s], kb, nb * TC_BN);
        tc_load_x<KPS>(st + C::W_BYTES, &tm_x, &full[s], kb, mb * MT);
      }
    }
  } else if (warp == 1) {
    pdl_wait();
    // MMA issuer (whole warp, one elected lane issues): accumulator buffer ui & 1 for the
    // ui-th unit of this CTA
    {
      constexpr uint32_t idesc = idesc_bf16(TC_MM, MT);
      uint32_t it = 0, ui = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < A.units; u += gridDim.x, ++ui) {
        const int nk = tc_unit(A, u, tiles).nk;
        const int ns = (nk + KPS - 1) / KPS, rot = u % ns;
        const uint32_t buf = (C::ACC_BUFS == 2) ? (ui & 1u) : 0u;
        const uint32_t use = (C::ACC_BUFS == 2) ? (ui >> 1) : ui;   // how often this buffer was used before
        if (ok && use >= 1 && !mbar_wait_w(&acc_empty[buf], (use - 1) & 1u, 104)) ok = false;
        tc_fence_after();
        const uint32_t d = tmem + buf * C::UNIT_COLS;
        for (int i = 0; i < ns; ++i, ++it) {
          const int s = it % C::STAGES;
          const uint32_t ph = (it / C::STAGES) & 1u;
          if (ok && !mbar_wait_w(&full[s], ph, 102)) ok = false;
          tc_fence_after();
          if (ok) {
            const uint32_t a0 = smem_u32(smem + s * C::STAGE_BYTES);
            const uint32_t b0 = a0 + C::W_BYTES;
            // k-blocks of this step that belong to the unit (the last step of an odd range
            // carries one k-block of the next range, or the zero fill past K: not multiplied)
            const int kv = min(KPS, nk - KPS * ((i + rot) % ns));
#pragma unroll
            for (int kk = 0; kk < KPS; ++kk) {
              if (kk < kv) {
#pragma unroll
                for (int q = 0; q < C::NACC; ++q)   // weight rows 128q..128q+127 → accumulator q
                  tc::umma4_bf16_warp(d + q * C::ACC_COLS,
                                      sdesc_sw128(a0 + kk * TC_BN * 128 + q * TC_MM * 128),
                                      sdesc_sw128(b0 + kk * MT * 128), idesc, (i > 0 || kk > 0) ? 1u : 0u);
              }
            }
          }
          tc::umma_commit_warp(&empty[s]);
        }
        tc::umma_commit_warp(&acc_full[buf]);
      }
    }
  } else {
    // epilogue: warp w reads TMEM lanes 32*(w%4)..+31, i.e. weight rows (output columns n)
    // 128q + 32*(w%4) + lane of accumulator q
    pdl_wait();
    const int quad = warp & 3;
    uint32_t ui = 0;
    for (int u = blockIdx.x; u < A.units; u += gridDim.x, ++ui) {
      const TcUnit U = tc_unit(A, u, tiles);
      const int mb = U.tile % A.m_tiles, nb = U.tile / A.m_tiles;
      const uint32_t buf = (C::ACC_BUFS == 2) ? (ui & 1u) : 0u;
      const uint32_t use = (C::ACC_BUFS == 2) ? (ui >> 1) : ui;
      const bool ok = mbar_wait(&acc_full[buf], use & 1u, 103);
      tc_fence_after();
      const bool split = A.splits > 1 || U.tail;
      // partial row / column of this unit (the tail has its own compact partial block)
      const int ldp = U.tail ? (A.n_tiles * A.m_tiles - A.full_units) * TC_BN : A.n_tiles * TC_BN;
      const int64_t prow0 = ((int64_t)U.slice * A.m_tiles + mb) * MT;
      const int pcol0 = U.tail ? (U.tile - A.full_units) * TC_BN : nb * TC_BN;
      if (split) {   // fp32 partial rows, one column per thread (coalesced across the warp)
#pragma unroll
        for (int q = 0; q < C::NACC; ++q) {
          float* prow = A.partial + prow0 * ldp + pcol0 + q * TC_MM + quad * 32 + lane;
          const uint32_t tbase = tmem + buf * C::UNIT_COLS + q * C::ACC_COLS + ((uint32_t)(quad * 32) << 16);
          for (int c0 = 0; c0 < MT; c0 += 32) {
            float v[32];
            tmem_ld32(tbase + c0, v);
            if (!ok) continue;
#pragma unroll
            for (int j = 0; j < 32; ++j) prow[(c0 + j) * ldp] = v[j];   // < 2^31: MT·ldp floats
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < C::NACC; ++q) {
          const int n = nb * TC_BN + q * TC_MM + quad * 32 + lane;
          const uint32_t tbase = tmem + buf * C::UNIT_COLS + q * C::ACC_COLS + ((uint32_t)(quad * 32) << 16);
          for (int c0 = 0; c0 < MT; c0 += 32) {
            float v[32];
            tmem_ld32(tbase + c0, v);
            if (!ok) continue;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const int m = mb * MT + c0 + j;
              if (m < A.m && n < A.n) {
                __nv_bfloat16* p = A.c + (int64_t)m * A.ldc + n;
                float r = dt<__nv_bfloat16>::round(v[j]);
                if (A.accumulate) r += __bfloat162float(*p);
                *p = __float2bfloat16_rn(r);
              }
            }
          }
        }
      }
      tc_fence_before();
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&acc_empty[buf])) : "memory");
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS)
                 : "memory");
  }
}

// ------------------------------------------------------------------ host side
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiled get_encode() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// 2-D bf16 row-major [rows, cols] with row stride ld (elements); box = [box_rows, 64 cols].
// The same row-major bf16 matrix viewed as [cols/64 k-blocks][rows][64 elements] (strides
// 128 B and ld·2 B; cols a multiple of 64): box = kps k-blocks × box_rows rows × 64 elements,
// laid out in shared memory k-block after k-block, each as 128B-swizzled K-major rows.
static bool make_map3(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                      int kps) {
  EncodeTiled enc = get_encode();
  if (!enc || cols % TC_BK != 0) return false;
  cuuint64_t dims[3] = {(cuuint64_t)TC_BK, (cuuint64_t)rows, (cuuint64_t)(cols / TC_BK)};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(TC_BK * 2)};
  cuuint32_t box[3] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows, (cuuint32_t)kps};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  EncodeTiled enc = get_encode();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)TC_BK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int pick_mt(int64_t m) {
  if (m <= 32) return 32;
  if (m <= 64) return 64;
  if (m <= 128) return 128;
  return 256;
}

struct TcPlan {
  int mt, bn, kps, m_tiles, n_tiles, n_kb, splits, kb_per_split;
  int full_units, tail_split, tail_kps;   // K-split tail of an unsplit plan (0: none)
  size_t partial_bytes;
};

// k-blocks per ring stage (TcCfg): 2 for 128-row units whose depth is a whole number of
// k-blocks (the 3-D TMA view needs K % 64 == 0) over at most 128 token rows, or over one tile
// of 256 token rows when the units take several rounds of the SMs (the vocabulary projection;
// with 256 rows a two-k-block stage is 96 KB, so the ring has two stages, which costs the split
// projections more than the larger boxes gain: measured 13.4 against 12.8 µs on 2048 × 4096,
// 170.8 against 174.5 µs on the vocabulary). 1 otherwise. QSP_GEMM_KPS=1 keeps one k-block per stage
// everywhere, =2 uses two wherever K allows (comparisons).
static int kps_for(int mt, int bn, int64_t k, bool multi_round) {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("QSP_GEMM_KPS");
    mode = e != nullptr ? atoi(e) : 0;
  }
  if (mode == 1 || bn != 128 || k % TC_BK != 0) return 1;
  return (mt <= 128 || mode == 2 || multi_round) ? 2 : 1;
}

// Split count: smallest estimated time over s in [1, 16], where one persistent CTA per SM
// walks ceil(units / SMs) units of ceil(k_blocks / s) k-blocks each, and a split pays for
// writing and merging s fp32 partials.
static TcPlan plan(int64_t m, int64_t n, int64_t k, int sm_count) {
  TcPlan p{};
  p.mt = pick_mt(m);
  p.m_tiles = (int)((m + p.mt - 1) / p.mt);
  // 256-row units when they fill the SMs in about one round (wide projections), 128-row
  // units otherwise (narrow outputs need many units; the vocabulary projection needs
  // double-buffered accumulators across ~8 units per SM)
  const int t256 = p.m_tiles * (int)((n + 255) / 256);
  p.bn = (t256 >= sm_count / 5 && t256 <= sm_count) ? 256 : 128;
  p.n_tiles = (int)((n + p.bn - 1) / p.bn);
  p.n_kb = (int)((k + TC_BK - 1) / TC_BK);
  const int tiles = p.m_tiles * p.n_tiles;
  p.kps = kps_for(p.mt, p.bn, k, p.m_tiles == 1 && tiles > sm_count);
  // µs per k-block per SM: ingest-bound (weight tile + activation tile at ~40 GB/s per SM)
  const double t_kb = (double)(p.bn + p.mt) * TC_BK * 2 / 40.0e3;
  double est[17] = {};
  double best = 1e30;
  for (int s = 1; s <= 16; ++s) {
    const int kps = (p.n_kb + s - 1) / s;
    const int ss = (p.n_kb + kps - 1) / kps;
    est[s] = 1e30;
    if (ss != s && s > 1) continue;
    const int units = tiles * ss;
    const int per_cta = (units + sm_count - 1) / sm_count;
    double t = per_cta * kps * t_kb + 1.0;
    if (ss > 1) t += 2.0 + (double)ss * p.m_tiles * p.mt * p.n_tiles * p.bn * 4.0 * 2.0 / 6.0e6;   // bytes / (6 TB/s)
    est[s] = t;
    best = std::min(best, t);
  }
  // the fewest splits within 3 % of the best estimate: fewer fp32 partials to write and merge
  // (measured: the 2048 × 6144 projection at 256 rows is 0.9 µs faster with 8 splits than 9)
  int best_s = 1;
  while (est[best_s] > 1.03 * best) ++best_s;
  p.kb_per_split = (p.n_kb + best_s - 1) / best_s;
  p.kb_per_split = (p.kb_per_split + p.kps - 1) / p.kps * p.kps;   // whole stages per split
  p.splits = (p.n_kb + p.kb_per_split - 1) / p.kb_per_split;
  p.partial_bytes = p.splits > 1 ? (size_t)p.splits * p.m_tiles * p.mt * p.n_tiles * p.bn * sizeof(float) : 0;
  // An unsplit plan whose tiles overrun whole rounds of the SMs by less than half a round
  // (the vocabulary projection: 1187 tiles on 148 SMs) would finish with a few CTAs computing
  // whole tiles while the rest idle. Those last tiles are split along K instead, so that
  // the last round takes a fraction of a tile's time.
  p.full_units = p.tail_split = p.tail_kps = 0;
  if (p.splits == 1 && p.m_tiles == 1) {
    const int grid = std::min(tiles, sm_count);
    const int full = tiles / grid * grid, r = tiles - full;
    if (tiles > grid && r > 0 && 2 * r <= grid) {
      int ts = std::min(std::min(16, p.n_kb / 2), grid / r);
      if (ts >= 2) {
        const int kps = ((p.n_kb + ts - 1) / ts + p.kps - 1) / p.kps * p.kps;
        p.full_units = full;
        p.tail_split = (p.n_kb + kps - 1) / kps;
        p.tail_kps = kps;
        p.partial_bytes = (size_t)p.tail_split * p.mt * r * p.bn * sizeof(float);
      }
    }
  }
  return p;
}

static int sm_count();
static int sm_count() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Sums `splits` fp32 partials [m, ldp] (split_stride floats apart, in split order) and applies
// the epilogue: c (+)= round(Σ); x += round(Σ) then RMSNorm into epi.y; or SwiGLU of the
// [gate | up] halves into epi.y.
int gemm_merge(const float* partial, int splits, int64_t split_stride, int ldp, __nv_bfloat16* c, int64_t ldc, int m,
               int n, int accumulate, const GemmEpi& epi, cudaStream_t st) {
  if (epi.kind == GEMM_EPI_RESNORM)
    return launch_pdl("qsp_gemm(split-k merge + residual + rmsnorm)", splitk_residual_rmsnorm_kernel, dim3(m),
                      dim3(RN_THREADS), 0, st, partial, splits, split_stride, ldp, c, ldc, epi.norm_w, epi.y, epi.ldy,
                      n, epi.eps);
  if (epi.kind == GEMM_EPI_SWIGLU) {
    const int inter = n / 2;
    dim3 g((unsigned)((inter / 4 + 255) / 256), (unsigned)m);
    return launch_pdl("qsp_gemm(split-k merge + swiglu)", splitk_swiglu_kernel, g, dim3(256), 0, st, partial, splits,
                      split_stride, ldp, epi.y, epi.ldy, inter);
  }
  dim3 rgrid((unsigned)((n / 4 + 255) / 256 + 1), (unsigned)m);
  return launch_pdl("qsp_gemm(split-k merge)", splitk_store_kernel, rgrid, dim3(256), 0, st, partial, splits,
                    split_stride, ldp, c, ldc, n, accumulate);
}

template <int MT, int BN, int KPS = 1>
static int launch_tc(const CUtensorMap& mw, const CUtensorMap& mx, const TcArgs& a, const TcPlan& p,
                     const GemmEpi& epi, cudaStream_t st) {
  auto kern = gemm_tc_kernel<MT, BN, KPS>;
  using TcCfgMT = TcCfg<MT, BN, KPS>;
  static bool attr_set = false;
  if (!attr_set) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)TcCfgMT::SMEM) != cudaSuccess)
      return set_error(QSP_ERR_CUDA, "qsp_gemm: cannot reserve %zu bytes of shared memory", TcCfgMT::SMEM);
    attr_set = true;
  }
  const int tiles = p.m_tiles * p.n_tiles;
  const int units = a.tail_split > 0 ? a.full_units + (tiles - a.full_units) * a.tail_split : tiles * p.splits;
  TcArgs aa = a;
  aa.m_tiles = p.m_tiles;
  aa.n_tiles = p.n_tiles;
  aa.units = units;
  const int grid = std::min(units, sm_count());
  int rc = launch_pdl("qsp_gemm(tcgen05)", kern, dim3(grid), dim3(TC_THREADS), TcCfgMT::SMEM, st, mw, mx, aa);
  if (rc) return rc;
  if (a.tail_split > 0) {   // the tail tiles' columns: c[:, full·BN, n)
    const int col0 = a.full_units * BN, nt = a.n - col0, ldp = (tiles - a.full_units) * BN;
    dim3 tgrid((unsigned)((nt / 4 + 255) / 256 + 1), (unsigned)a.m);
    return launch_pdl("qsp_gemm(k-split tail merge)", splitk_store_kernel, tgrid, dim3(256), 0, st,
                      (const float*)a.partial, a.tail_split, (int64_t)MT * ldp, ldp, a.c + col0, a.ldc, nt,
                      a.accumulate);
  }
  if (p.splits == 1) return rc;
  const int ldp = p.n_tiles * BN;
  return gemm_merge(a.partial, p.splits, (int64_t)p.m_tiles * MT * ldp, ldp, a.c, a.ldc, a.m, a.n, a.accumulate, epi,
                    st);
}

static size_t ws_need(const TcPlan& p) { return p.partial_bytes; }

size_t gemm_tc_workspace(int64_t m, int64_t n, int64_t k) { return ws_need(plan(m, n, k, sm_count())); }

// Returns QSP_ERR_UNSUPPORTED when the operands cannot go through TMA (alignment) or the
// workspace is too small for the chosen split; the caller then uses the CUDA-core kernel.
// `split_out` (optional) reports whether the product went through a split-K merge (which
// then already applied `epi`); otherwise c holds the stored product and the caller applies
// the epilogue with the standalone kernels.
int gemm_tc(const void* a, int64_t lda, const void* w, int64_t ldw, void* c, int64_t ldc, int64_t m, int64_t n,
            int64_t k, int flags, void* workspace, size_t ws_bytes, cudaStream_t st, const GemmEpi* epi_in,
            int* split_out) {
  GemmEpi epi{};
  if (epi_in) epi = *epi_in;
  if (split_out) *split_out = 0;
  if (!aligned(a, 16) || !aligned(w, 16) || (lda * 2) % 16 != 0 || (ldw * 2) % 16 != 0 || k % 8 != 0)
    return QSP_ERR_UNSUPPORTED;
  TcPlan p = plan(m, n, k, sm_count());
  if (p.splits > 1) {
    if (workspace == nullptr || ws_bytes < ws_need(p)) {
      p.splits = 1;  // no room for partials: one K range per tile
      p.kb_per_split = p.n_kb;
      p.partial_bytes = 0;
    }
  }
  if (p.splits > 1 && !aligned(workspace, 256)) return QSP_ERR_UNSUPPORTED;
  if (p.tail_split > 0 && (workspace == nullptr || ws_bytes < ws_need(p) || !aligned(workspace, 256)))
    p.tail_split = 0;   // no room for the tail partials: whole tiles to the end
  if (p.splits > 1 && epi.kind == GEMM_EPI_RESNORM && n > RN_MAXV * RN_THREADS * 4) return QSP_ERR_UNSUPPORTED;
  if (p.splits > 1 && epi.kind != GEMM_EPI_STORE && (n % 8) != 0) return QSP_ERR_UNSUPPORTED;
  CUtensorMap mw, mx;
  if (p.kps == 2) {
    if (!make_map3(&mw, w, n, k, ldw, p.bn, 2) || !make_map3(&mx, a, m, k, lda, p.mt, 2)) return QSP_ERR_UNSUPPORTED;
  } else if (!make_map(&mw, w, n, k, ldw, p.bn) || !make_map(&mx, a, m, k, lda, p.mt)) {
    return QSP_ERR_UNSUPPORTED;
  }
  TcArgs args{};
  args.c = static_cast<__nv_bfloat16*>(c);
  args.ldc = ldc;
  args.m = (int)m;
  args.n = (int)n;
  args.n_kb = p.n_kb;
  args.kb_per_split = p.kb_per_split;
  args.splits = p.splits;
  args.accumulate = (flags & QSP_GEMM_ACCUMULATE) ? 1 : 0;
  if (p.splits > 1 || p.tail_split > 0) args.partial = static_cast<float*>(workspace);
  args.full_units = p.tail_split > 0 ? p.full_units : 0;
  args.tail_split = p.tail_split;
  args.tail_kps = p.tail_kps;
  if (split_out) *split_out = p.splits > 1;
  const bool wide = p.bn == 256;
  if (p.kps == 2) {
    switch (p.mt) {
      case 32: return launch_tc<32, 128, 2>(mw, mx, args, p, epi, st);
      case 64: return launch_tc<64, 128, 2>(mw, mx, args, p, epi, st);
      case 128: return launch_tc<128, 128, 2>(mw, mx, args, p, epi, st);
      default: return launch_tc<256, 128, 2>(mw, mx, args, p, epi, st);
    }
  }
  switch (p.mt) {
    case 32: return wide ? launch_tc<32, 256>(mw, mx, args, p, epi, st) : launch_tc<32, 128>(mw, mx, args, p, epi, st);
    case 64: return wide ? launch_tc<64, 256>(mw, mx, args, p, epi, st) : launch_tc<64, 128>(mw, mx, args, p, epi, st);
    case 128:
      return wide ? launch_tc<128, 256>(mw, mx, args, p, epi, st) : launch_tc<128, 128>(mw, mx, args, p, epi, st);
    default:
      return wide ? launch_tc<256, 256>(mw, mx, args, p, epi, st) : launch_tc<256, 128>(mw, mx, args, p, epi, st);
  }
}

}  // namespace qsp

namespace qsp {
int gdn_device_error(int reset);
int attn_device_error(int reset);
int moe_device_error(int reset);
int gemm_cl_device_error(int reset);
int gemm_pair_device_error(int reset);
int core_device_error(int reset);
int sample_device_error(int reset);
int probe_device_error(int reset);
}

extern "C" int qsp_device_status(int32_t* code, int32_t reset) {
  QSP_REQUIRE(code != nullptr, "qsp_device_status: null pointer");
  const int gdn = qsp::gdn_device_error(reset);
  const int attn = qsp::attn_device_error(reset);
  const int moe = qsp::moe_device_error(reset);
  const int cl = qsp::gemm_cl_device_error(reset);
  const int others[] = {qsp::gemm_pair_device_error(reset), qsp::core_device_error(reset),
                        qsp::sample_device_error(reset), qsp::probe_device_error(reset)};
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, qsp::g_qsp_dev_error, sizeof(int));
  if (e != cudaSuccess) return qsp::set_error(QSP_ERR_CUDA, "qsp_device_status: %s", cudaGetErrorString(e));
  *code = v != 0 ? v : (gdn != 0 ? gdn : (attn != 0 ? attn : (moe != 0 ? moe : cl)));
  for (int o : others)
    if (*code == 0) *code = o;
  if (reset && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(qsp::g_qsp_dev_error, &zero, sizeof(int));
    if (e != cudaSuccess) return qsp::set_error(QSP_ERR_CUDA, "qsp_device_status: %s", cudaGetErrorString(e));
  }
  return QSP_OK;
}

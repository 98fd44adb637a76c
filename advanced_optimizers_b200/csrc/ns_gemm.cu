// Newton–Schulz GEMM for sm_100a: D = bf16(alpha * (A @ B) + beta * C)
//
// A persistent kernel: each CTA (one per SM) walks the 128 x 256 output
// tiles t = blockIdx.x, blockIdx.x + gridDim.x, ... with 5th-generation
// tensor cores and two accumulators in tensor memory, so the epilogue of one
// tile overlaps the main loop of the next:
//   * warp 0 (one elected lane) streams 128x64 A and 256x64 B tiles into a
//     4-stage shared-memory ring with TMA (cp.async.bulk.tensor, 128-byte
//     swizzle, no multicast), completing on "full" mbarriers;
//   * warp 1 owns the tensor memory (2 x 256 fp32 columns x 128 lanes); one
//     elected lane issues tcgen05.mma (kind::f16, bf16 in, fp32 accumulate),
//     four K=16 steps per stage, commits each stage to its "empty" mbarrier
//     and each finished tile to its accumulator's "full" mbarrier;
//   * warps 2..5 wait for an accumulator, read it with tcgen05.ld (each warp
//     its 32-lane quarter of the tile's rows), write bf16(alpha*acc + beta*C)
//     and release the accumulator on its "empty" mbarrier.
// A is K-major ([M][K], K contiguous).  B is K-major ([N][K]) or N-major
// ([K][N], N contiguous) — the latter is how X enters X' = a X + B X.
// Every wait is bounded and also gives up when another role has; the CTA
// then drains its tensor-core work (bounded), frees its tensor memory,
// reports through *err and returns.
//
// Newton–Schulz itself (Muon_util.py:7-121): per iteration
//   quintic: A = X X^T;  B = b A + c A A;  X = a X + B X
//   CANS:    A = X X^T;  X = c1 X + c3 A X
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdio>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "advopt.h"
#include "capi_internal.h"
#include "common.cuh"

namespace advopt {
namespace ns {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int B_BYTES = BN * BK * 2;            // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
constexpr int THREADS = 192;
constexpr uint32_t TMEM_COLS = 256;

// ---- descriptors ----
// Shared-memory matrix descriptor (tcgen05): start address, leading / stride
// byte offsets (>> 4), version 1, 128-byte swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;          // version = 1 (sm_100)
  d |= (uint64_t)2 << 61;          // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: bf16 A/B, fp32 D, M=128, N=256.
__host__ __device__ constexpr uint32_t instr_desc(bool b_mn_major) {
  return (1u << 4)                 // D format f32
         | (1u << 7)               // A bf16
         | (1u << 10)              // B bf16
         | (0u << 15)              // A K-major
         | ((b_mn_major ? 1u : 0u) << 16)
         | ((uint32_t)(BN >> 3) << 17)
         | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct GemmArgs {
  uint16_t* D;
  const uint16_t* C;
  int ldd, ldc;
  int M, N, K;
  float alpha, beta;
  int32_t* err;
  int sym;   // D is symmetric (M == N): compute the blocks on or above the diagonal, mirror the rest
};

// Origin of tile t of a CTA's walk.  General: m-fastest over the M/BM x N/BN
// grid.  Symmetric output: only the BN x BN blocks on or above the diagonal,
// column block nb holding row tiles 0 .. 2nb+1 (still m-fastest, so the
// concurrent tiles share B column blocks); the epilogue writes each
// off-diagonal block twice, as itself and transposed.
__device__ __forceinline__ void tile_origin(int t, int n_mb, int sym, int& m0, int& n0) {
  if (!sym) {
    m0 = (t % n_mb) * BM;
    n0 = (t / n_mb) * BN;
    return;
  }
  int nb = 0;
  while ((nb + 1) * (nb + 2) <= t) ++nb;
  m0 = (t - nb * (nb + 1)) * BM;
  n0 = nb * BN;
}

constexpr uint32_t TMEM_ALLOC = 2 * TMEM_COLS;   // two accumulators

// Bounded wait that also gives up once another role of the CTA has.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t i = 0; i < (1u << 22); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *abort_flag) return false;
  }
  return false;
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__global__ void __launch_bounds__(THREADS, 1)
    ns_gemm_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapB, GemmArgs g,
                   int b_mn_major) {
  extern __shared__ unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle atoms
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full_bar[STAGES], empty_bar[STAGES], acc_full[2], acc_empty[2], drain;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  volatile int* abort_v = &abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ktiles = g.K / BK;
  const int n_nb = g.N / BN;
  const int n_mb = g.M / BM;
  // walked m-fastest: concurrent tiles share B column blocks
  const int ntiles = g.sym ? n_nb * (n_nb + 1) : n_mb * n_nb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(&drain, 1);
    abort_flag = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                 "r"(TMEM_ALLOC)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      uint32_t it = 0;
      for (int t = blockIdx.x; t < ntiles && !*abort_v; t += gridDim.x) {
        int m0, n0;
        tile_origin(t, n_mb, g.sym, m0, n0);
        for (int kt = 0; kt < ktiles; ++kt, ++it) {
          const int s = (int)(it % STAGES);
          const uint32_t use = it / STAGES;
          if (use > 0 && !wait_or_abort(&empty_bar[s], (use - 1) & 1u, abort_v)) {
            abort_flag = 1;
            break;
          }
          unsigned char* sa = smem + s * STAGE_BYTES;
          unsigned char* sb = sa + A_BYTES;
          mbar_arrive_tx(&full_bar[s], STAGE_BYTES);
          tma_load_2d(sa, &mapA, kt * BK, m0, &full_bar[s]);
          if (b_mn_major) {
            // B tile = 4 boxes of [64 k-rows][64 n-cols], each 8 KB
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 8192, &mapB, n0 + 64 * j, kt * BK, &full_bar[s]);
          } else {
            tma_load_2d(sb, &mapB, kt * BK, n0, &full_bar[s]);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    if (lane == 0) {
      const uint32_t idesc = instr_desc(b_mn_major != 0);
      uint32_t it = 0;
      int i = 0;
      for (int t = blockIdx.x; t < ntiles && !*abort_v; t += gridDim.x, ++i) {
        const int acc = i & 1;
        const uint32_t use = (uint32_t)i >> 1;
        if (use > 0 && !wait_or_abort(&acc_empty[acc], (use - 1) & 1u, abort_v)) {
          abort_flag = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d_tmem = tmem + (uint32_t)acc * TMEM_COLS;
        bool ok = true;
        for (int kt = 0; kt < ktiles; ++kt, ++it) {
          const int s = (int)(it % STAGES);
          if (!wait_or_abort(&full_bar[s], (it / STAGES) & 1u, abort_v)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            // A K-major: 16 elements = 32 bytes along the swizzled row
            const uint64_t ad = smem_desc(sa + k * 32, 16, 1024);
            const uint64_t bd = b_mn_major ? smem_desc(sb + k * 2048, 8192, 1024)   // 2 groups of 8 k-rows per step
                                           : smem_desc(sb + k * 32, 16, 1024);
            mma_bf16(d_tmem, ad, bd, idesc, (kt > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty_bar[s]);
        }
        if (!ok) {
          abort_flag = 1;
          break;
        }
        mma_commit(&acc_full[acc]);
      }
    }
  } else {
    // ---- epilogue: warps 2..5, TMEM lane quarter = warp % 4 ----
    const int quarter = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
      const int acc = i & 1;
      const uint32_t use = (uint32_t)i >> 1;
      if (!wait_or_abort(&acc_full[acc], use & 1u, abort_v)) {
        abort_flag = 1;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      int m0, n0;
      tile_origin(t, n_mb, g.sym, m0, n0);
      const bool mirror = g.sym && (m0 / BN) < (n0 / BN);   // off-diagonal block of a symmetric D
      const int row = m0 + quarter * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)acc * TMEM_COLS;
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tmem_ld16(taddr + c, r);
        const int col = n0 + c;
        float cv[16];
        if (g.beta != 0.0f && g.C) {
          const uint4* cp = reinterpret_cast<const uint4*>(g.C + (size_t)row * g.ldc + col);
          const uint4 c0 = __ldg(cp), c1 = __ldg(cp + 1);
          const uint32_t w[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            cv[2 * q] = __uint_as_float(w[q] << 16);
            cv[2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 16; ++q) cv[q] = 0.0f;
        }
        uint32_t o[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float v0 = __fmaf_rn(g.alpha, __uint_as_float(r[2 * q]), __fmul_rn(g.beta, cv[2 * q]));
          const float v1 = __fmaf_rn(g.alpha, __uint_as_float(r[2 * q + 1]), __fmul_rn(g.beta, cv[2 * q + 1]));
          o[q] = f_to_bf16_rne(v0) | (f_to_bf16_rne(v1) << 16);
        }
        uint4* dp = reinterpret_cast<uint4*>(g.D + (size_t)row * g.ldd + col);
        dp[0] = make_uint4(o[0], o[1], o[2], o[3]);
        dp[1] = make_uint4(o[4], o[5], o[6], o[7]);
        if (mirror) {
          // D[col + j][row]: the 32 lanes hold consecutive rows, so each
          // column store of the warp is 64 contiguous bytes
          uint16_t* dt = g.D + (size_t)col * g.ldd + row;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            dt[(size_t)(2 * q) * g.ldd] = (uint16_t)(o[q] & 0xFFFFu);
            dt[(size_t)(2 * q + 1) * g.ldd] = (uint16_t)(o[q] >> 16);
          }
        }
      }
      // the accumulator has been read: the MMA warp may overwrite it
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      mbar_arrive(&acc_empty[acc]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (abort_flag) {
    // drain: wait (bounded) for every tensor-core op issued so far before the
    // tensor memory is released
    if (threadIdx.x == 32) {
      mma_commit(&drain);
      mbar_wait(&drain, 0);
    }
    if (threadIdx.x == 0 && g.err) atomicExch(g.err, 1);
    __syncthreads();
  }
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_ALLOC) : "memory");
  }
}

// ---- host: tensor maps ----
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode ? ADVOPT_OK : set_error(ADVOPT_E_CUDA, "cuTensorMapEncodeTiled is unavailable");
}

// 2-D bf16 tensor map: rows x cols row-major with leading dimension ld
// (elements); box = box_cols x box_rows, 128-byte swizzle.
int encode_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols,
               uint32_t box_rows) {
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {ld * 2};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(ADVOPT_E_INVALID, "cuTensorMapEncodeTiled rejected a Newton-Schulz operand");
  return ADVOPT_OK;
}

// The chain's operands are the same workspace buffers step after step, so
// their tensor maps are encoded once and kept (a host-side cache keyed by
// every encoding argument; cleared when it grows past 4096 entries).
struct MapKey {
  uintptr_t base;
  uint64_t rows, cols, ld;
  uint32_t box_cols, box_rows;
  bool operator==(const MapKey& o) const {
    return base == o.base && rows == o.rows && cols == o.cols && ld == o.ld && box_cols == o.box_cols &&
           box_rows == o.box_rows;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    uint64_t h = k.base * 0x9E3779B97F4A7C15ull;
    h ^= (k.rows * 0xC2B2AE3D27D4EB4Full) + (h << 6) + (h >> 2);
    h ^= (k.cols * 0x165667B19E3779F9ull) + (h << 6) + (h >> 2);
    h ^= (k.ld + ((uint64_t)k.box_cols << 32 | k.box_rows)) + (h << 6) + (h >> 2);
    return (size_t)h;
  }
};

int make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_cols,
             uint32_t box_rows) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{reinterpret_cast<uintptr_t>(base), rows, cols, ld, box_cols, box_rows};
  {
    std::lock_guard<std::mutex> lock(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *map = it->second;
      return ADVOPT_OK;
    }
  }
  const int rc = encode_map(map, base, rows, cols, ld, box_cols, box_rows);
  if (rc != ADVOPT_OK) return rc;
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *map);
  return ADVOPT_OK;
}

}  // namespace ns
}  // namespace advopt

using namespace advopt;

namespace advopt {
namespace ns {
// sym: the caller guarantees D is symmetric (A @ B symmetric and C symmetric
// or unused); only the blocks on or above the diagonal are computed.
int launch_gemm(void* D, int32_t ldd, const void* A, int32_t lda, const void* B, int32_t ldb, int32_t b_mn_major,
                const void* C, int32_t ldc, int32_t M, int32_t N, int32_t K, float alpha, float beta, int32_t* err,
                void* stream, int32_t sym = 0) {
  if (!D || !A || !B || M <= 0 || N <= 0 || K <= 0)
    return set_error(ADVOPT_E_INVALID, "advopt_ns_gemm: null operand or empty shape");
  if (M % BM || N % BN || K % BK)
    return set_error(ADVOPT_E_INVALID, "advopt_ns_gemm: M must be a multiple of 128, N of 256, K of 64");
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) | reinterpret_cast<uintptr_t>(D)) & 15 ||
      (C && (reinterpret_cast<uintptr_t>(C) & 15)) || lda % 8 || ldb % 8 || ldd % 8 || (C && ldc % 8))
    return set_error(ADVOPT_E_INVALID, "advopt_ns_gemm: operands must be 16-byte aligned with ld % 8 == 0");
  if (beta != 0.0f && !C) return set_error(ADVOPT_E_INVALID, "advopt_ns_gemm: beta != 0 needs C");
  if (sym && (M != N || M % BN)) return set_error(ADVOPT_E_INVALID, "advopt_ns_gemm: a symmetric D needs M == N, a multiple of 256");
  int rc = get_encode();
  if (rc != ADVOPT_OK) return rc;
  CUtensorMap ma, mb;
  rc = make_map(&ma, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, BK, BM);
  if (rc != ADVOPT_OK) return rc;
  if (b_mn_major) rc = make_map(&mb, B, (uint64_t)K, (uint64_t)N, (uint64_t)ldb, 64, BK);
  else rc = make_map(&mb, B, (uint64_t)N, (uint64_t)K, (uint64_t)ldb, BK, BN);
  if (rc != ADVOPT_OK) return rc;
  GemmArgs g;
  g.D = static_cast<uint16_t*>(D);
  g.C = static_cast<const uint16_t*>(C);
  g.ldd = ldd;
  g.ldc = ldc;
  g.M = M;
  g.N = N;
  g.K = K;
  g.alpha = alpha;
  g.beta = beta;
  g.err = err;
  g.sym = sym ? 1 : 0;
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(ns_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return check_cuda(attr_err, "advopt_ns_gemm: smem attribute");
  static int sms = 0;
  if (sms == 0) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
      sms = 148;
  }
  {
    const int ntiles = sym ? (N / BN) * (N / BN + 1) : (M / BM) * (N / BN);
    const int grid = ntiles < sms ? ntiles : sms;
    ns_gemm_kernel<<<grid, THREADS, SMEM_BYTES, static_cast<cudaStream_t>(stream)>>>(ma, mb, g, b_mn_major);
  }
  return check_cuda(cudaGetLastError(), "advopt_ns_gemm");
}
}  // namespace ns
}  // namespace advopt

extern "C" int advopt_ns_gemm(void* D, int32_t ldd, const void* A, int32_t lda, const void* B, int32_t ldb,
                              int32_t b_mn_major, const void* C, int32_t ldc, int32_t M, int32_t N, int32_t K,
                              float alpha, float beta, int32_t* err, void* stream) {
  return advopt::ns::launch_gemm(D, ldd, A, lda, B, ldb, b_mn_major, C, ldc, M, N, K, alpha, beta, err, stream);
}

// Same GEMM with a symmetric output: only the 256 x 256 blocks of D on or
// above the diagonal are computed, and each off-diagonal block is stored a
// second time, transposed, below the diagonal (the X X^T and b A + c A A
// products of the quintic iteration, Muon_util.py:108-112).
extern "C" int advopt_ns_gemm_sym(void* D, int32_t ldd, const void* A, int32_t lda, const void* B, int32_t ldb,
                                  int32_t b_mn_major, const void* C, int32_t ldc, int32_t M, int32_t K, float alpha,
                                  float beta, int32_t* err, void* stream) {
  return advopt::ns::launch_gemm(D, ldd, A, lda, B, ldb, b_mn_major, C, ldc, M, M, K, alpha, beta, err, stream, 1);
}

// The whole Newton–Schulz chain on a loaded workspace (Muon_util.py:7-121):
// quintic (a, b, c) or CANS with coefficients from the singular-value bounds
// starting at [cns_lower_bound, 1] (Muon_util.py:69-105), computed here in
// double precision exactly as the reference's Python does.
extern "C" int advopt_ns_chain(void* x, void* c, void* a, void* b, int32_t m_pad, int32_t n_pad, int32_t steps,
                               int32_t cns, double coef_a, double coef_b, double coef_c, double cns_lower_bound,
                               void** final_x, int32_t* err, void* stream) {
  using advopt::ns::launch_gemm;
  if (!x || !c || !a || (!cns && !b) || !final_x || steps < 0 || m_pad <= 0 || n_pad <= 0)
    return advopt::set_error(ADVOPT_E_INVALID, "advopt_ns_chain: bad arguments");
  int rc = ADVOPT_OK;
  if (cns) {
    double lb = cns_lower_bound, ub = 1.0;
    for (int i = 0; i < steps && rc == ADVOPT_OK; ++i) {
      const double lb_ub = lb * ub;
      const double e_sq = (lb * lb + lb_ub + ub * ub) / 3.0;
      const double kk = 2.0 * std::pow(e_sq, 1.5);
      const double ll = lb_ub * (lb + ub);
      const double den = kk + ll;
      const double alpha = 6.0 / den;
      const double c1 = alpha * e_sq, c3 = -alpha / 3.0;
      rc = launch_gemm(a, m_pad, x, n_pad, x, n_pad, 0, nullptr, 0, m_pad, m_pad, n_pad, 1.0f, 0.0f, err, stream, 1);
      if (rc == ADVOPT_OK)
        rc = launch_gemm(c, n_pad, a, m_pad, x, n_pad, 1, x, n_pad, m_pad, n_pad, m_pad, (float)c3, (float)c1, err,
                         stream);
      std::swap(x, c);
      const double e = (kk - ll) / den;
      lb = 1.0 - e;
      ub = 1.0 + e;
    }
  } else {
    for (int i = 0; i < steps && rc == ADVOPT_OK; ++i) {
      // A = X X^T and B = b A + c A A are symmetric: upper blocks only
      rc = launch_gemm(a, m_pad, x, n_pad, x, n_pad, 0, nullptr, 0, m_pad, m_pad, n_pad, 1.0f, 0.0f, err, stream, 1);
      if (rc == ADVOPT_OK)
        rc = launch_gemm(b, m_pad, a, m_pad, a, m_pad, 1, a, m_pad, m_pad, m_pad, m_pad, (float)coef_c, (float)coef_b,
                         err, stream, 1);
      if (rc == ADVOPT_OK)
        rc = launch_gemm(c, n_pad, b, m_pad, x, n_pad, 1, x, n_pad, m_pad, n_pad, m_pad, 1.0f, (float)coef_a, err,
                         stream);
      std::swap(x, c);
    }
  }
  *final_x = x;
  return rc;
}


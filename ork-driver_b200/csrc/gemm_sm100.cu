// gemm_sm100.cu -- batched-M matmul on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// C[M][N] = A[M][K] . W[N][K]^T with both operands K-major (the activations as given, the weight in its
// resident [N][K] layout). One CTA computes a 128 x TN output tile:
//   warp 0      TMA producer: 2-D tiled bulk-tensor loads of a 128 x 128-byte A tile and a TN x 128-byte
//               W tile per K block into a STAGES-deep shared-memory ring (128-byte swizzle, the UMMA
//               canonical K-major layout), completion tracked by mbarrier transaction counts;
//   warp 1      allocates TN TMEM columns; one thread issues tcgen05.mma (kind::i8 -> s32, or
//               kind::f16 -> f32) per 32-byte K step, and tcgen05.commit frees each stage and finally
//               signals the epilogue;
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns at a time from their TMEM sub-partition and
//               store the int32 / fp32 row segment to C.
// Integer accumulation in TMEM is exact int32, so results equal ork-driver's CPU oracle bit for bit.
// Out-of-range rows / K columns are zero-filled by the tensor map, so M, N and K need no padding
// beyond the API's own alignment rules.
//
// Every mbarrier wait is bounded by a clock deadline; on expiry the kernel records an error in a
// device flag that the host checks, and all roles fall through to the common exit (no hang).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "ork_internal.h"

namespace orkb {

__device__ unsigned int g_tc_error = 0;

namespace {

constexpr int BM = 128;          // MMA M (rows of A per tile)
constexpr int BK_BYTES = 128;    // K bytes per stage (one 128-byte swizzle row)
constexpr uint64_t kWaitCycles = 4000000000ull;  // ~2 s at 1.9 GHz

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

// Bounded wait for the phase with the given parity; false (and the error flag set) on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > kWaitCycles) {
      atomicOr(&g_tc_error, 1u);
      return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major tile with 128-byte swizzle: rows of 128 bytes, 8-row
// core-matrix groups 1024 bytes apart (stride byte offset), leading byte offset unused (1), descriptor
// version 1 (sm_100), layout type 2 (SWIZZLE_128B). The tile base must be 1024-byte aligned.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor: kind::i8 (signed x signed -> s32) or kind::f16 (f16 x f16 -> f32), both
// operands K-major, M = 128, N = TN.
template <bool F16>
__host__ __device__ constexpr uint32_t idesc(int tn) {
  return (F16 ? (1u << 4) : (2u << 4))        // D format: f32 / s32
         | (F16 ? 0u : (1u << 7))             // A format: f16 / signed int8
         | (F16 ? 0u : (1u << 10))            // B format: f16 / signed int8
         | ((uint32_t)(tn >> 3) << 17)        // N >> 3
         | ((uint32_t)(BM >> 4) << 24);       // M >> 4
}

template <bool F16>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t id, uint32_t accum) {
  if constexpr (F16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(accum));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(accum));
  }
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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
}

template <bool F16, int TN, int STAGES>
__global__ void __launch_bounds__(192, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap mapA, const __grid_constant__ CUtensorMap mapW, void *__restrict__ Cout,
               int M, int N, int K) {
  constexpr uint32_t A_BYTES = BM * BK_BYTES;
  constexpr uint32_t W_BYTES = TN * BK_BYTES;
  constexpr int ESZ = F16 ? 2 : 1;
  constexpr int KSTEPS = BK_BYTES / 32;  // 32-byte MMA K steps per stage (K=32 int8 / K=16 f16)
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *sA = smem;
  uint8_t *sW = smem + STAGES * A_BYTES;
  uint64_t *bars = (uint64_t *)(sW + STAGES * W_BYTES);  // full[STAGES], empty[STAGES], done
  uint32_t *tmem_slot = (uint32_t *)(bars + 2 * STAGES + 1);

  asm volatile("griddepcontrol.launch_dependents;");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * TN, m0 = blockIdx.y * BM;
  const int KB = (K * ESZ + BK_BYTES - 1) / BK_BYTES;
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES), done = smem_u32(bars + 2 * STAGES);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mapA) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mapW) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int kb = 0; kb < KB; kb++) {
        const int s = kb % STAGES;
        const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) break;
        mbar_expect_tx(full0 + 8 * s, A_BYTES + W_BYTES);
        const int x = kb * (BK_BYTES / ESZ);
        tma_load_2d(smem_u32(sA + s * A_BYTES), &mapA, x, m0, full0 + 8 * s);
        tma_load_2d(smem_u32(sW + s * W_BYTES), &mapW, x, n0, full0 + 8 * s);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id = idesc<F16>(TN);
      bool ok = true;
      for (int kb = 0; kb < KB && ok; kb++) {
        const int s = kb % STAGES;
        const uint32_t ph = (uint32_t)(kb / STAGES) & 1u;
        ok = mbar_wait(full0 + 8 * s, ph);
        if (!ok) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t ad = sw128_desc(smem_u32(sA + s * A_BYTES));
        const uint64_t wd = sw128_desc(smem_u32(sW + s * W_BYTES));
#pragma unroll
        for (int k = 0; k < KSTEPS; k++)  // advance 32 bytes (2 x 16-byte units) along K within the row
          umma<F16>(tmem, ad + 2 * k, wd + 2 * k, id, (kb | k) != 0);
        umma_commit(empty0 + 8 * s);
      }
      umma_commit(done);
    }
  } else {
    // epilogue: warps 2..5 -> TMEM sub-partitions (warp % 4)
    const int sub = warp & 3;
    const int row = sub * 32 + lane;
    const int m = m0 + row;
    const bool ok = mbar_wait(done, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < TN; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(sub * 32) << 16) + (uint32_t)c0, r);
        if (m < M) {
          uint32_t *dst = (uint32_t *)Cout + (size_t)m * N + n0 + c0;
#pragma unroll
          for (int q = 0; q < 8; q++)
            if (n0 + c0 + 4 * q < N)
              *reinterpret_cast<uint4 *>(dst + 4 * q) = make_uint4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TN));
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void *p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (PFN_cuTensorMapEncodeTiled_v12000)p;
  });
  return fn;
}

// 2-D map over a row-major [rows][cols] matrix of esz-byte elements; box = box_rows x 128 bytes, SW128.
bool make_map(CUtensorMap *map, const void *base, int rows, int cols, int esz, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * esz};
  const cuuint32_t box[2] = {(cuuint32_t)(BK_BYTES / esz), (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, esz == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
                        const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool F16, int TN, int STAGES>
cudaError_t launch_tc(const RunArgs &a, cudaStream_t s, bool pdl) {
  constexpr int ESZ = F16 ? 2 : 1;
  CUtensorMap mA, mW;
  if (!make_map(&mA, a.A, a.M, a.K, ESZ, BM) || !make_map(&mW, a.W, a.N, a.K, ESZ, TN)) return cudaErrorInvalidValue;
  constexpr size_t smem = 1024 + (size_t)STAGES * (BM + TN) * BK_BYTES + (2 * STAGES + 1) * 8 + 16;
  auto kern = gemm_tc_kernel<F16, TN, STAGES>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    attr_set = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.N + TN - 1) / TN, (a.M + BM - 1) / BM);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, mA, mW, a.C, a.M, a.N, a.K);
}

}  // namespace

bool gemm_tc_supports(int fmt, int M, int K, int N) {
  (void)K;
  if (fmt != FMT_I8 && fmt != FMT_F16) return false;
  if (N % 16) return false;
  return M >= 1 && encode_fn() != nullptr;
}

cudaError_t launch_gemm_tc(const RunArgs &a, cudaStream_t s, bool pdl, int *launches) {
  if ((uintptr_t)a.A % 16 || (uintptr_t)a.W % 16 || (uintptr_t)a.C % 16) return cudaErrorMisalignedAddress;
  cudaError_t e;
  if (a.fmt == FMT_I8) e = launch_tc<false, 128, 6>(a, s, pdl);
  else if (a.fmt == FMT_F16) e = launch_tc<true, 128, 6>(a, s, pdl);
  else return cudaErrorNotSupported;
  if (e == cudaSuccess && launches) ++*launches;
  return e;
}

unsigned int tc_error_flag(bool reset) {
  unsigned int v = 0;
  cudaMemcpyFromSymbol(&v, g_tc_error, sizeof v);
  if (reset && v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_tc_error, &z, sizeof z);
  }
  return v;
}

}  // namespace orkb

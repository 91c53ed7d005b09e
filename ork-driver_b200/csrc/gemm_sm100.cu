// gemm_sm100.cu -- matmul on the 5th-generation tensor cores (tcgen05), sm_100a.
//
// C[M][N] = A[M][K] . W[N][K]^T with both operands K-major (the activations as given, the weight in its
// resident [N][K] layout). A CTA owns a 128 x TN tile of the MMA's D = R . S^T, where the 128-row
// operand R and the TN-row operand S are either (A, W) or, for small M ("swap", M <= 64), (W, A): the
// weight then fills the 128-row side and the activations the narrow side, so decode-sized M wastes no
// MMA rows. Roles inside a CTA (192 threads):
//   warp 0      TMA producer: 2-D tiled bulk-tensor loads of a 128 x 128-byte R tile and a TN x 128-byte
//               S tile per K block into a STAGES-deep ring (128-byte swizzle, the UMMA canonical K-major
//               layout); completion tracked by mbarrier transaction counts;
//   warp 1      allocates the TMEM accumulator; one thread issues tcgen05.mma (kind::i8 -> s32, or
//               kind::f16 -> f32) per 32-byte K step; tcgen05.commit frees each stage and finally
//               signals the epilogue;
//   warps 2..5  epilogue: tcgen05.ld from their TMEM sub-partition into 128-byte-swizzled staging
//               boxes in the (now idle) ring, written to C by bulk tensor stores (the TMA).
// Split-K across a thread-block cluster: the SK CTAs of a cluster (gridDim.z = cluster z = SK) take
// consecutive K ranges of the same tile. Integer tiles: split 0 zeroes the tile, a split-phase cluster
// barrier orders that before any partial lands, and every split's partial is reduce-added into C by the
// TMA (cp.reduce.async.bulk.tensor .add: the int32 sum is exact in any order, so results equal
// ork-driver's CPU oracle bit for bit). fp32 tiles (fp16 weights) are summed in a fixed order through
// distributed shared memory instead, so their result does not depend on which split finishes first.
// Out-of-range rows / K columns are zero-filled by the tensor maps, so M, N and K need no padding.
//
// Every mbarrier wait is bounded by a clock deadline; on expiry the kernel records an error in a
// device flag that the host checks, and all roles fall through to the common exit (no hang).
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <mutex>

#include "nibble.cuh"
#include "errword.cuh"
#include "ork_internal.h"

namespace orkb {

__device__ unsigned int g_tc_error = 0;

namespace {

constexpr int BM = 128;                          // MMA M: rows of the R operand per tile
constexpr int BK_BYTES = 128;                    // K bytes per stage (one 128-byte swizzle row)
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
      { atomicOr(&g_tc_error, 1u); err_word_set(); }
      return false;
    }
  }
}

// L2 prefetch of one tile of a tensor map (no data returned, no effect on the values later loads read)
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y) : "memory");
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
  return (F16 ? (1u << 4) : (2u << 4))   // D format: f32 / s32
         | (F16 ? 0u : (1u << 7))        // A format: f16 / signed int8
         | (F16 ? 0u : (1u << 10))       // B format: f16 / signed int8
         | ((uint32_t)(tn >> 3) << 17)   // N >> 3
         | ((uint32_t)(BM >> 4) << 24);  // M >> 4
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

// 32 lanes x 16 columns without waiting: several loads are put in flight and completed by one
// tmem_wait_ld(), so the TMEM read latency is paid once per batch instead of once per 16 columns. The
// destination registers must not be touched before the wait.
__device__ __forceinline__ void tmem_ld16_nowait(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- TMA epilogue: C leaves the CTA as bulk tensor stores, or -- for split-K integer tiles -- as bulk
// tensor reduce-adds into C, which the L2 sums exactly in any order ---------------------------------------
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, int x, int y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(map), "r"(x),
               "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap *map, int x, int y, uint32_t src) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   map),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// every bulk store / reduce this thread issued has read its shared-memory source
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

// One warp's 32 accumulator rows (TN columns from TMEM address taddr) through its staging boxes to C:
// box b holds columns 32b..32b+31 as 32 rows of 128 bytes, row = lane, with the 16-byte chunk q of a row
// at position q ^ (row & 7) -- the tensor map's 128-byte swizzle, which makes these row-per-lane writes
// free of bank conflicts. Box b lies at sbox + b * 16 KB (the four epilogue warps' boxes interleave:
// warp w's box b at (4b + w) * 4 KB of the tile's staging). Boxes go in groups of up to four (128
// columns: one TMEM wait, one proxy fence, then one TMA store -- or, for split-K integer tiles,
// reduce-add -- per box at C columns x0 + 32b, rows y), so the TMA drains one group while the next is
// written.
template <int TN>
__device__ __forceinline__ void drain_rows_tma(uint32_t taddr, int lane, uint32_t sbox, const CUtensorMap *mapC,
                                               int x0, int y, int M, int N, bool reduce) {
  static_assert(TN % 32 == 0, "row tiles drain in 32-column boxes");
  constexpr int NB = TN / 32;                                          // boxes
  constexpr int GB = NB % 4 == 0 ? 4 : NB % 3 == 0 ? 3 : NB % 2 == 0 ? 2 : 1;  // boxes per group
  const uint32_t rowoff = (uint32_t)lane * 128u, sw = (uint32_t)(lane & 7);
#pragma unroll 1
  for (int g = 0; g < NB; g += GB) {
    uint32_t v[2 * GB][16];
#pragma unroll
    for (int j = 0; j < 2 * GB; j++) tmem_ld16_nowait(taddr + (uint32_t)(32 * g + 16 * j), v[j]);
    tmem_wait_ld();
#pragma unroll
    for (int k = 0; k < GB; k++) {
      const uint32_t box = sbox + (uint32_t)(g + k) * 16384u + rowoff;
#pragma unroll
      for (int q = 0; q < 4; q++) {
        st_shared_v4(box + ((q ^ sw) << 4), v[2 * k][4 * q], v[2 * k][4 * q + 1], v[2 * k][4 * q + 2],
                     v[2 * k][4 * q + 3]);
        st_shared_v4(box + (((q + 4) ^ sw) << 4), v[2 * k + 1][4 * q], v[2 * k + 1][4 * q + 1],
                     v[2 * k + 1][4 * q + 2], v[2 * k + 1][4 * q + 3]);
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> the TMA (async proxy)
    __syncwarp();
    if (lane == 0 && y < M) {
#pragma unroll
      for (int k = 0; k < GB; k++)
        if (x0 + 32 * (g + k) < N) {
          const uint32_t box = sbox + (uint32_t)(g + k) * 16384u;
          if (reduce) tma_reduce_add_2d(mapC, x0 + 32 * (g + k), y, box);
          else tma_store_2d(mapC, x0 + 32 * (g + k), y, box);
        }
      bulk_commit();
    }
  }
}

// Swapped tiles hold a column of C per lane (TMEM lane = weight row n, columns = activation rows m): the
// warp's TN x 32 block goes to staging as [TN rows m][32 words n] (consecutive lanes, consecutive words:
// no bank conflicts), one TMA box of 32 x TN. Columns go 64 at a time.
template <int TN>
__device__ __forceinline__ void drain_cols_tma(uint32_t taddr, int lane, uint32_t sbox) {
  constexpr int CB = TN < 64 ? TN : 64;
  constexpr int NJ = CB / 16;
#pragma unroll 1
  for (int cb = 0; cb < TN; cb += CB) {
    uint32_t v[NJ][16];
#pragma unroll
    for (int j = 0; j < NJ; j++) tmem_ld16_nowait(taddr + (uint32_t)(cb + 16 * j), v[j]);
    tmem_wait_ld();
#pragma unroll
    for (int j = 0; j < NJ; j++)
#pragma unroll
      for (int q = 0; q < 16; q++)
        asm volatile("st.shared.u32 [%0], %1;" ::"r"(sbox + (uint32_t)(((cb + 16 * j + q) * 32 + lane) * 4)),
                     "r"(v[j][q])
                     : "memory");
  }
}
// Epilogue store of a 32-row x 32-column block held one row per lane: the warp transposes it through
// its own shared-memory tile (row stride 36 words: both the row-per-lane writes and the row-wise reads
// are free of bank conflicts) so that every global store instruction writes four whole 128-byte rows
// of C instead of 32 scattered 16-byte pieces.
constexpr int kStgStride = 36;
__device__ __forceinline__ void store_rows32(uint32_t *stg, const uint32_t (&lo)[16], const uint32_t (&hi)[16],
                                             uint32_t *C, int M, int N, int m0, int n0, int lane) {
#pragma unroll
  for (int k = 0; k < 16; k += 4) {
    *reinterpret_cast<uint4 *>(stg + lane * kStgStride + k) = make_uint4(lo[k], lo[k + 1], lo[k + 2], lo[k + 3]);
    *reinterpret_cast<uint4 *>(stg + lane * kStgStride + 16 + k) = make_uint4(hi[k], hi[k + 1], hi[k + 2], hi[k + 3]);
  }
  __syncwarp();
  const int ch = lane & 7, n = n0 + 4 * ch;
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const int r = 4 * j + (lane >> 3), m = m0 + r;
    const uint4 x = *reinterpret_cast<const uint4 *>(stg + r * kStgStride + 4 * ch);
    if (m < M && n < N) *reinterpret_cast<uint4 *>(C + (size_t)m * N + n) = x;
  }
  __syncwarp();
}

// Drains one warp's 32 TMEM lanes (TN accumulator columns from taddr) into C, or into the split-K
// partial tile P. Loads are batched (up to 128 columns in flight, one wait). Non-swapped tiles hold a
// row of C per lane and are stored through the warp's staging tile; swapped tiles hold a column of C
// per lane (lanes along n), which stores coalesced as is. gr0 = global R row of lane 0, c0 = global
// origin of the S columns, prow = this lane's row in the partial tile.
template <bool SWAP, int TN, int PSTR>
__device__ __forceinline__ void drain_rows(uint32_t taddr, int lane, bool split, uint32_t *P, int prow,
                                           uint32_t *stg, uint32_t *C, int M, int N, int gr0, int c0) {
  constexpr int CB = TN % 128 == 0 ? 128 : TN % 64 == 0 ? 64 : TN % 32 == 0 ? 32 : 16;  // divides TN
  constexpr int NJ = CB / 16;
#pragma unroll 1
  for (int cb = 0; cb < TN; cb += CB) {
    uint32_t v[NJ][16];
#pragma unroll
    for (int j = 0; j < NJ; j++) tmem_ld16_nowait(taddr + (uint32_t)(cb + 16 * j), v[j]);
    tmem_wait_ld();
    if (split) {
#pragma unroll
      for (int j = 0; j < NJ; j++) {
        const int cc = cb + 16 * j;
        if constexpr (SWAP) {
#pragma unroll
          for (int q = 0; q < 16; q++) P[(cc + q) * PSTR + prow] = v[j][q];
        } else {
#pragma unroll
          for (int q = 0; q < 16; q += 4)
            *reinterpret_cast<uint4 *>(P + prow * PSTR + cc + q) =
                make_uint4(v[j][q], v[j][q + 1], v[j][q + 2], v[j][q + 3]);
        }
      }
    } else if constexpr (SWAP) {  // D[n][m] -> C[m][n]
      const int n = gr0 + lane;
      if (n < N) {
#pragma unroll
        for (int j = 0; j < NJ; j++)
#pragma unroll
          for (int q = 0; q < 16; q++) {
            const int m = c0 + cb + 16 * j + q;
            if (m < M) C[(size_t)m * N + n] = v[j][q];
          }
      }
    } else {
      static_assert(NJ % 2 == 0, "row stores go in 32-column blocks");
#pragma unroll
      for (int j = 0; j < NJ; j += 2) store_rows32(stg, v[j], v[j + 1], C, M, N, gr0, c0 + cb + 16 * j, lane);
    }
  }
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// the two halves of a cluster barrier, for threads that can signal long before they need the others
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }

// Split-K zeroing ordered by a per-tile flag in global memory instead of a cluster barrier (so the
// splits of a tile need not share a cluster): word 0 = the tile is zeroed, word 1 = splits that have
// seen it. Split 0 sets word 0 once its zeroes are written; every other split waits for it (bounded)
// before its first reduce-add; each split counts itself in word 1 once past that point, and the last
// one clears both words, so the flags are zero again when the launch completes (a later launch reads
// them only after its dependency wait, i.e. after this grid has finished).
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }  // warps 2..5
__device__ __forceinline__ void tile_flag_count(unsigned int *tf, int SK) {
  if (atomicAdd(&tf[1], 1u) == (unsigned int)(SK - 1)) {
    tf[1] = 0u;
    tf[0] = 0u;
  }
}
__device__ __forceinline__ void tile_flag_set(unsigned int *tf) {
  asm volatile("fence.acq_rel.gpu;\n\tst.relaxed.gpu.global.u32 [%0], 1;" ::"l"(tf) : "memory");
}
__device__ __forceinline__ bool tile_flag_wait(const unsigned int *tf);
// a non-zero split's epilogue warps (0..127 = ct): split 0's zeroes of this launch are in C from here on
__device__ __forceinline__ void tile_flag_pass(const unsigned int *tf, int ct) {
  asm volatile("griddepcontrol.wait;" ::: "memory");  // a flag read only once earlier launches are done
  if (ct == 0) tile_flag_wait(tf);
  epi_bar_sync();
}
__device__ __forceinline__ bool tile_flag_wait(const unsigned int *tf) {
  const uint64_t t0 = clock64();
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(tf) : "memory");
    if (v) return true;
    if (clock64() - t0 > kWaitCycles) {
      { atomicOr(&g_tc_error, 1u); err_word_set(); }
      return false;
    }
    __nanosleep(32);
  }
}

__device__ __forceinline__ uint4 ld_cluster_v4(uint32_t cluster_addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

template <bool F16>
__device__ __forceinline__ uint4 add4(uint4 a, uint4 b);

// Split-K reduction of this CTA's share of a tile after the cluster barrier: output items t = first,
// first + stride, ... < items, an item being one 16-byte vector of C (output row t / vpr, vector t % vpr
// of the tile, C row m0 + row, column n0 + 4 * vector). The SK partial tiles lie at the same offset of
// the shared memory of cluster ranks rank0 + rstep * q. Items go BATCH at a time and every remote read
// of a batch is issued before its first add, so a thread waits out one distributed-shared-memory round
// trip per batch rather than one per item (one per item was several microseconds of every split launch).
template <bool F16, int SK>
__device__ __forceinline__ void reduce_split(uint32_t pbase, int pstr, int first, int stride, int items, int vpr,
                                             uint32_t rank0, uint32_t rstep, uint32_t *C, int N, int m0, int n0) {
  constexpr int BATCH = SK <= 2 ? 8 : SK <= 4 ? 4 : 2;
  uint32_t remote[SK];
#pragma unroll
  for (int q = 0; q < SK; q++) {
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote[q]) : "r"(pbase), "r"(rank0 + rstep * q));
  }
  for (int t0 = first; t0 < items; t0 += BATCH * stride) {
    uint4 v[BATCH][SK];
#pragma unroll
    for (int b = 0; b < BATCH; b++) {
      const int t = t0 + b * stride;
      if (t < items) {
        const uint32_t off = (uint32_t)((t / vpr) * pstr + 4 * (t % vpr)) * 4u;
#pragma unroll
        for (int q = 0; q < SK; q++) v[b][q] = ld_cluster_v4(remote[q] + off);
      }
    }
#pragma unroll
    for (int b = 0; b < BATCH; b++) {
      const int t = t0 + b * stride;
      if (t < items) {
        uint4 acc = v[b][0];
#pragma unroll
        for (int q = 1; q < SK; q++) acc = add4<F16>(acc, v[b][q]);
        *reinterpret_cast<uint4 *>(C + (size_t)(m0 + t / vpr) * N + n0 + 4 * (t % vpr)) = acc;
      }
    }
  }
}

template <bool F16>
__device__ __forceinline__ void reduce_split_any(int SK, uint32_t pbase, int pstr, int first, int stride, int items,
                                                 int vpr, uint32_t rank0, uint32_t rstep, uint32_t *C, int N, int m0,
                                                 int n0) {
  switch (SK) {
    case 2: reduce_split<F16, 2>(pbase, pstr, first, stride, items, vpr, rank0, rstep, C, N, m0, n0); break;
    case 3: reduce_split<F16, 3>(pbase, pstr, first, stride, items, vpr, rank0, rstep, C, N, m0, n0); break;
    case 4: reduce_split<F16, 4>(pbase, pstr, first, stride, items, vpr, rank0, rstep, C, N, m0, n0); break;
    case 5: reduce_split<F16, 5>(pbase, pstr, first, stride, items, vpr, rank0, rstep, C, N, m0, n0); break;
    case 6: reduce_split<F16, 6>(pbase, pstr, first, stride, items, vpr, rank0, rstep, C, N, m0, n0); break;
    case 7: reduce_split<F16, 7>(pbase, pstr, first, stride, items, vpr, rank0, rstep, C, N, m0, n0); break;
    default: reduce_split<F16, 8>(pbase, pstr, first, stride, items, vpr, rank0, rstep, C, N, m0, n0); break;
  }
}

template <bool F16>
__device__ __forceinline__ uint4 add4(uint4 a, uint4 b) {
  if constexpr (F16) {
    return make_uint4(__float_as_uint(__uint_as_float(a.x) + __uint_as_float(b.x)),
                      __float_as_uint(__uint_as_float(a.y) + __uint_as_float(b.y)),
                      __float_as_uint(__uint_as_float(a.z) + __uint_as_float(b.z)),
                      __float_as_uint(__uint_as_float(a.w) + __uint_as_float(b.w)));
  } else {
    return make_uint4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
  }
}

// Expands one stage's nibble tile (WROWS rows x 64 bytes) into the 128-byte-swizzled int8 MMA tile
// (row r, 16-byte k chunk c at chunk position c ^ (r & 7)): WROWS * 8 chunks over the 128 converter
// threads. Every nibble word of the thread's chunks is loaded before the first expansion, so the
// chunks' integer chains overlap: the four converter warps of a CTA have little else to hide their
// latency with, and with a 2-chunk unroll the expansion, not the weight stream, set the pace of
// decode-sized nibble runs (ncu: 41 % issue-active, stalls on fixed-latency dependencies).
template <int FMT, int WROWS, int CT = 128>
__device__ __forceinline__ void expand_stage(const uint8_t *src, uint8_t *dst, int ct, const Nf4Tables &tb) {
  static_assert((WROWS * 8) % CT == 0 && (CT / 8) % 8 == 0, "whole chunks per converter thread");
  constexpr int ITEMS = WROWS * 8 / CT;
  constexpr int RSTEP = CT / 8;        // rows between a thread's chunks (a multiple of 8: same swizzle)
  const int r0 = ct >> 3, c = ct & 7;  // chunk q of this thread: row r0 + RSTEP q, same k chunk c
  const uint32_t s_src = smem_u32(src) + (uint32_t)(r0 * 64 + c * 8);
  const uint32_t s_dst = smem_u32(dst) + (uint32_t)(r0 * 128 + ((c ^ (r0 & 7)) << 4));
  uint32_t nb[ITEMS][2];
#pragma unroll
  for (int q = 0; q < ITEMS; q++)
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];"
                 : "=r"(nb[q][0]), "=r"(nb[q][1])
                 : "r"(s_src + (uint32_t)(q * RSTEP * 64)));
#pragma unroll
  for (int q = 0; q < ITEMS; q++) {
    const uint2 lo = expand8<FMT>(nb[q][0], tb), hi = expand8<FMT>(nb[q][1], tb);
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(s_dst + (uint32_t)(q * RSTEP * 128)), "r"(lo.x),
                 "r"(lo.y), "r"(hi.x), "r"(hi.y)
                 : "memory");
  }
}

// Converter warps of the one-CTA kernel: nibble weights in row tiles get four more warps (6..9 beside
// the epilogue's 2..5), so each SM sub-partition runs two converter warps and one hides the other's
// dependent-latency stalls (w4a8 6144x2048 M256 10.8 -> 10.4 us, M32 6.4 -> 6.0-6.3). Decode-sized
// (swapped) grids already put two to four CTAs, each with its four converter warps, on an SM; eight
// there were slower (70B NF4 M = 8: 686 -> 650 tok/s) and they keep four.
template <int FMT, bool SWAP>
constexpr int conv_warps() { return ((FMT == FMT_U4 || FMT == FMT_NF4) && !SWAP) ? 8 : 4; }
template <int FMT, bool SWAP>
constexpr int tc_threads() { return 64 + 32 * conv_warps<FMT, SWAP>(); }

constexpr int tmem_cols(int tn) { return tn <= 32 ? 32 : tn <= 64 ? 64 : tn <= 128 ? 128 : 256; }

// Nibble weights (FMT_U4 / FMT_NF4): the W tile arrives as nibbles ([rows][64 bytes] per 128-k block)
// in a staging buffer and the four epilogue warps, idle during the main loop, expand it in registers
// (expand8, nibble.cuh) into the 128-byte-swizzled int8 tile the MMA reads, then publish it to the async
// proxy.
template <int FMT, bool SWAP, int TN, int STAGES, int NA>
__global__ void __launch_bounds__(tc_threads<FMT, SWAP>())
gemm_tc_kernel(const __grid_constant__ CUtensorMap mapR, const __grid_constant__ CUtensorMap mapS,
               const __grid_constant__ CUtensorMap mapC, void *__restrict__ Cout, int M, int N, int K,
               Nf4Tables tb, unsigned int *__restrict__ tflag, int prew) {
  // NA accumulators of 128 rows stacked along the R side (TM = 128*NA): each K step issues NA MMAs that
  // share the S tile, so S is fetched once per 128*NA rows (less operand traffic per output)
  constexpr bool F16 = FMT == FMT_F16;
  constexpr bool NIB = FMT == FMT_U4 || FMT == FMT_NF4;
  constexpr int TM = BM * NA;
  constexpr int WROWS = SWAP ? TM : TN;                 // rows of the weight tile
  constexpr uint32_t R_BYTES = TM * BK_BYTES;
  constexpr uint32_t S_BYTES = TN * BK_BYTES;
  constexpr uint32_t NIB_BYTES = NIB ? WROWS * 64 : 0;  // nibble staging per stage
  // bytes the TMA delivers per stage: the activation tile, and the weight tile (int8/f16) or nibbles
  constexpr uint32_t TX_BYTES = NIB ? ((SWAP ? S_BYTES : R_BYTES) + NIB_BYTES) : (R_BYTES + S_BYTES);
  constexpr int ESZ = F16 ? 2 : 1;                      // activation element size
  constexpr int KSTEPS = BK_BYTES / 32;                 // 32-byte MMA K steps per stage
  constexpr int TCOLS = tmem_cols(TN * NA);
  constexpr int PSTR = SWAP ? (TM + 4) : (TN + 4);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *sR = smem;
  uint8_t *sS = smem + STAGES * R_BYTES;
  uint8_t *sN = sS + STAGES * S_BYTES;                   // nibble staging (NIB only)
  uint64_t *bars = (uint64_t *)(sN + STAGES * NIB_BYTES);  // full[S], empty[S], conv[S], done
  uint32_t *tmem_slot = (uint32_t *)(bars + 3 * STAGES + 1);
  uint32_t *P = (uint32_t *)smem;
  uint8_t *sW = SWAP ? sR : sS;                          // where the MMA reads the weight tile

  asm volatile("griddepcontrol.launch_dependents;");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * TM, c0 = blockIdx.y * TN;
  const int SK = gridDim.z, ks = blockIdx.z;
  const int KB = (K * ESZ + BK_BYTES - 1) / BK_BYTES;
  const int kb0 = (int)((long long)KB * ks / SK), kb1 = (int)((long long)KB * (ks + 1) / SK);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES), conv0 = smem_u32(bars + 2 * STAGES),
                 done = smem_u32(bars + 3 * STAGES);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
      mbar_init(conv0 + 8 * s, conv_warps<FMT, SWAP>());  // one arrival per converter warp
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mapR) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mapS) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  // weight tile load of stage s for k block kb (int8/f16 straight into the MMA tile; nibbles to staging)
  auto load_w = [&](int s, int kb) {
    if constexpr (NIB) {
      tma_load_2d(smem_u32(sN + s * NIB_BYTES), SWAP ? &mapR : &mapS, kb * 64, SWAP ? r0 : c0, full0 + 8 * s);
    } else {
      const int x = kb * (BK_BYTES / ESZ);
      if (SWAP) tma_load_2d(smem_u32(sR + s * R_BYTES), &mapR, x, r0, full0 + 8 * s);
      else tma_load_2d(smem_u32(sS + s * S_BYTES), &mapS, x, c0, full0 + 8 * s);
    }
  };
  auto load_a = [&](int s, int kb) {
    const int x = kb * (BK_BYTES / ESZ);
    if (SWAP) tma_load_2d(smem_u32(sS + s * S_BYTES), &mapS, x, c0, full0 + 8 * s);
    else tma_load_2d(smem_u32(sR + s * R_BYTES), &mapR, x, r0, full0 + 8 * s);
  };
  auto prefetch_a = [&](int kb) {
    const int x = kb * (BK_BYTES / ESZ);
    if (SWAP) tma_prefetch_2d(&mapS, x, c0);
    else tma_prefetch_2d(&mapR, x, r0);
  };

  bool ep_ok = false;  // the epilogue warps' accumulator is complete (no bounded wait expired)
  // integer split-K: the splits reduce-add into C after split 0 has zeroed it. A split-phase cluster
  // barrier orders the two: every thread arrives as early as it can (split 0's epilogue warps once the
  // zeroes are written) and only the epilogue warps wait, well before they need to -- or, with tile
  // flags (the splits then are not one cluster), split 0 sets the tile's flag and the others wait on it
  const bool tma_reduce = !F16 && SK > 1;
  const bool flagz = tma_reduce && tflag != nullptr;
  unsigned int *tf = flagz ? tflag + 2 * (blockIdx.y * gridDim.x + blockIdx.x) : nullptr;
  // every thread of the cluster arrives once: here warps 0-1 and the converter-only warps 6-9 (and all
  // warps of the other splits); split 0's epilogue warps after their zeroes
  if (tma_reduce && !flagz && (warp < 2 || warp >= 6 || ks != 0)) cluster_arrive();
  if (warp == 0) {
    if (lane == 0) {
      // the weight tiles do not depend on the previous kernel: the first ring's worth is requested
      // before waiting on it (programmatic dependent launch); activations only after the wait
      // the first `pre` stages' weight tiles are requested before the wait; after it the activation
      // tiles go first, then the rest of the first ring (both tiles of a stage)
      const int ring = (kb1 - kb0) < STAGES ? (kb1 - kb0) : STAGES;
      const int pre = prew < ring ? prew : ring;
      for (int i = 0; i < pre; i++) {
        mbar_expect_tx(full0 + 8 * i, TX_BYTES);
        load_w(i, kb0 + i);
      }
      // the first ring's activation tiles are prefetched into L2 before the wait (a hint: the loads
      // after it read the current data through L2 either way), so a cold A costs L2 latency, not HBM's.
      // Every CTA of a row (column, when swapped) of tiles reads the same A tiles: one CTA in eight of a
      // swapped grid asks, and for row tiles only the first weight tile's CTAs (each tile once: a
      // prefetch by all 16-48 CTAs sharing it slowed M = 512 runs by 3-4 %)
      if (SWAP ? (blockIdx.x & 7) == 0 : blockIdx.y == 0)
        for (int i = 0; i < ring; i++) prefetch_a(kb0 + i);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int i = 0; i < pre; i++) load_a(i, kb0 + i);
      for (int i = pre; i < ring; i++) {
        mbar_expect_tx(full0 + 8 * i, TX_BYTES);
        load_a(i, kb0 + i);
        load_w(i, kb0 + i);
      }
      for (int kb = kb0 + ring; kb < kb1; kb++) {
        const int i = kb - kb0, s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) break;
        mbar_expect_tx(full0 + 8 * s, TX_BYTES);
        load_w(s, kb);
        load_a(s, kb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t id = idesc<F16>(TN);
      for (int kb = kb0; kb < kb1; kb++) {
        const int i = kb - kb0, s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait((NIB ? conv0 : full0) + 8 * s, ph)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t rd = sw128_desc(smem_u32(sR + s * R_BYTES));
        const uint64_t sd = sw128_desc(smem_u32(sS + s * S_BYTES));
#pragma unroll
        for (int k = 0; k < KSTEPS; k++)  // advance 32 bytes (2 x 16-byte units) along K within the row
#pragma unroll
          for (int a = 0; a < NA; a++)    // accumulator a: R rows 128a.., TMEM columns a*TN..
            umma<F16>(tmem + (uint32_t)(a * TN), rd + (uint64_t)(a * (BM * BK_BYTES >> 4)) + 2 * k, sd + 2 * k, id,
                      (kb > kb0 || k > 0) ? 1u : 0u);
        umma_commit(empty0 + 8 * s);
      }
      umma_commit(done);
    }
  } else {
    const int ct = threadIdx.x - 64;  // over the converter warps 2.. (0..127: warps 2..5, the epilogue's)
    const bool epi = warp < 6;        // warps 6..9 (nibble weights only) convert and then leave
    if (epi && tma_reduce && ks == 0) {
      // split 0 zeroes the tile of C that every split reduce-adds into, once the previous grid (which may
      // still read C) has finished
      asm volatile("griddepcontrol.wait;" ::: "memory");
      const int rows = SWAP ? min(TN, M - c0) : min(TM, M - r0);
      const int cols = SWAP ? min(TM, N - r0) : min(TN, N - c0);
      const int m0 = SWAP ? c0 : r0, n0 = SWAP ? r0 : c0, vpr = cols / 4;
      uint32_t *Cz = (uint32_t *)Cout;
      for (int t = ct; t < rows * vpr; t += 128)
        *reinterpret_cast<uint4 *>(Cz + (size_t)(m0 + t / vpr) * N + n0 + 4 * (t % vpr)) = make_uint4(0, 0, 0, 0);
      asm volatile("fence.proxy.async.global;" ::: "memory");  // the zeroes, before any reduce (async proxy)
      __syncwarp();
      if (flagz) {
        epi_bar_sync();  // all four warps' zeroes are written
        if (ct == 0) tile_flag_set(tf);
      } else {
        cluster_arrive();
      }
    }
    // the other splits wait for the flag now, while their accumulators fill (nibble weights: after the
    // conversion, which these warps do meanwhile); they count themselves once their adds are issued
    if (!NIB && epi && flagz && ks != 0) tile_flag_pass(tf, ct);
    if constexpr (NIB) {
      // converter: per stage, WROWS x 8 chunks of 16 output bytes (row r, k chunk c), written at the
      // 128-byte-swizzle position (chunk c ^ (r & 7)) of the 1024-byte-aligned tile
      bool cok = true;
      for (int kb = kb0; kb < kb1 && cok; kb++) {
        const int i = kb - kb0, s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        cok = mbar_wait(full0 + 8 * s, ph);
        if (!cok) break;
        const uint8_t *src = sN + s * NIB_BYTES;
        uint8_t *dst = sW + s * (SWAP ? R_BYTES : S_BYTES);
        expand_stage<FMT, WROWS, 32 * conv_warps<FMT, SWAP>()>(src, dst, ct, tb);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic writes -> async proxy
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(conv0 + 8 * s) : "memory");
      }
    }
    if (!epi) {
      // converter-only warps: nothing more to do
    } else {
    if (tma_reduce) {  // split 0's zeroes are visible to this thread's reduces from here on
      if (flagz) {
        if (NIB && ks != 0) tile_flag_pass(tf, ct);
      } else {
        __syncwarp();
        cluster_wait();
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    // epilogue warps 2..5 read TMEM sub-partition (warp % 4): TMEM lane = row of an R accumulator. The
    // ring is idle once done fired and holds the staging boxes (or, for fp16 split-K, the partial tile)
    const int sub = warp & 3;
    ep_ok = mbar_wait(done, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ep_ok) {
      if (F16 && SK > 1) {
        uint32_t *stg = (uint32_t *)smem + sub * 32 * kStgStride;
#pragma unroll 1
        for (int a = 0; a < NA; a++)
          drain_rows<SWAP, TN, PSTR>(tmem + ((uint32_t)(sub * 32) << 16) + (uint32_t)(a * TN), lane, true, P,
                                     a * BM + sub * 32 + lane, stg, (uint32_t *)Cout, M, N, r0 + a * BM + sub * 32,
                                     c0);
      } else if constexpr (SWAP) {
        const uint32_t sbox = smem_u32(smem) + (uint32_t)(sub * TN * 128);
        drain_cols_tma<TN>(tmem + ((uint32_t)(sub * 32) << 16), lane, sbox);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0 && r0 + sub * 32 < N && c0 < M) {
          if (tma_reduce) tma_reduce_add_2d(&mapC, r0 + sub * 32, c0, sbox);
          else tma_store_2d(&mapC, r0 + sub * 32, c0, sbox);
          bulk_commit();
        }
      } else {
#pragma unroll 1
        for (int a = 0; a < NA; a++)
          drain_rows_tma<TN>(tmem + ((uint32_t)(sub * 32) << 16) + (uint32_t)(a * TN), lane,
                             smem_u32(smem) + (uint32_t)(((a * (TN / 32)) * 4 + sub) * 4096), &mapC, c0,
                             r0 + a * BM + sub * 32, M, N, tma_reduce);
      }
    }
    if (flagz && ct == 0) tile_flag_count(tf, SK);  // past the flag (or its setter): the last one clears it
    }  // epi
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  if (F16 && SK > 1) {
    cluster_sync();  // every CTA's partial tile is in its shared memory
    {
      // fp16 (fp32 C): the partials are summed through distributed shared memory in a fixed order, so the
      // result does not depend on the order the splits finish in
      const int out_rows = SWAP ? min(TN, M - c0) : min(TM, M - r0);
      const int out_cols = SWAP ? min(TM, N - r0) : min(TN, N - c0);
      const int vpr = out_cols / 4;  // N is a multiple of 16, tiles start at multiples of 16
      const int items = out_rows > 0 && out_cols > 0 ? out_rows * vpr : 0;
      reduce_split_any<F16>(SK, smem_u32(P), PSTR, ks * 192 + (int)threadIdx.x, SK * 192, items, vpr, 0u, 1u,
                            (uint32_t *)Cout, N, SWAP ? c0 : r0, SWAP ? r0 : c0);
      cluster_sync();  // no CTA leaves while its partial tile may still be read
    }
  }
  // the staging boxes have been read by the TMA before the CTA (and its shared memory) goes; the writes
  // themselves complete with the grid
  if (warp >= 2 && lane == 0) bulk_wait_read();
  __syncthreads();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
}

// ---------------------------------------------------------------------------------------------------
// CTA-pair variant (tcgen05 cta_group::2). Two CTAs of a cluster (ranks 2j, 2j+1: the "pair") compute
// one 256 x TN tile of D = R . S^T with M = 256 MMAs issued by the even CTA (the leader). Each CTA holds
// its own 128 rows of R and its own TN/2 rows of S in shared memory and its own 128 rows of D (all TN
// columns) in TMEM; the MMA reads the operand halves of both CTAs. Per output a CTA therefore loads
// (128 + TN/2) rows instead of (128 + TN) -- the L2-to-SM operand stream, which bounds this kernel on
// B200 (~45-60 GB/s per SM), shrinks by a third at TN = 256 compared with the one-CTA 128 x 256 tile.
// Every load is issued by the CTA that owns the destination; there is no multicast.
//   loads   int8/f16: both operands of both CTAs complete on the leader's full[s] barrier (the
//           cta_group::2 form of the tiled TMA load, which may signal the peer CTA's barrier); the
//           leader expects both CTAs' bytes. Nibble weights land in the owner's staging buffer and
//           complete on its own wfull[s]; its converter warps then arrive on the leader's conv[s].
//   mma     the leader waits full[s] (and conv[s]), issues the MMAs, and commits to the empty[s]
//           barriers of both CTAs, and finally to both done barriers.
//   epilog  each CTA drains its own TMEM rows; split-K partial tiles reduce across the SK CTAs that
//           hold the same pair half (cluster ranks half + 2q) through distributed shared memory.
// A cluster-wide barrier after initialisation guarantees that no peer signals a barrier or the MMA
// writes a TMEM allocation that does not exist yet; another one before the end keeps both CTAs (their
// shared memory and TMEM) alive until the pair is done.

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t mapa_u32(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  return remote;
}

// tiled load into this CTA's shared memory whose completion is counted on a barrier of either CTA of
// the pair (bar: shared::cluster address)
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

template <bool F16>
__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t id,
                                          uint32_t accum) {
  if constexpr (F16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(accum));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(id), "r"(accum));
  }
}

// completion of this thread's pair MMAs, signalled on one barrier (shared::cluster address, either CTA)
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// bounded wait with cluster-scope acquire (for arrivals made by the peer CTA's threads)
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = clock64();
  while (true) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (clock64() - t0 > kWaitCycles) {
      { atomicOr(&g_tc_error, 1u); err_word_set(); }
      return false;
    }
  }
}

template <bool F16>
__host__ __device__ constexpr uint32_t idesc_pair(int tn) {
  return (idesc<F16>(tn) & ~(0x1Fu << 24)) | ((uint32_t)(256 >> 4) << 24);  // M = 256
}

template <int FMT, bool SWAP, int TN, int STAGES>
__global__ void __launch_bounds__(192)
gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap mapR, const __grid_constant__ CUtensorMap mapS,
                    const __grid_constant__ CUtensorMap mapC, void *__restrict__ Cout, int M, int N, int K,
                    Nf4Tables tb, unsigned int *__restrict__ tflag, int prew) {
  constexpr bool F16 = FMT == FMT_F16;
  constexpr bool NIB = FMT == FMT_U4 || FMT == FMT_NF4;
  constexpr int HS = TN / 2;                             // S rows held by each CTA
  constexpr int WROWS = SWAP ? BM : HS;                  // weight rows held by each CTA
  constexpr uint32_t R_BYTES = BM * BK_BYTES;
  constexpr uint32_t S_BYTES = HS * BK_BYTES;
  constexpr uint32_t NIB_BYTES = NIB ? WROWS * 64 : 0;
  constexpr uint32_t A_BYTES = SWAP ? S_BYTES : R_BYTES;  // activation tile per CTA and stage
  // bytes counted on the leader's full[s] per stage (both CTAs): A and W, or A alone for nibbles
  constexpr uint32_t FULL_TX = 2 * (NIB ? A_BYTES : (R_BYTES + S_BYTES));
  constexpr int ESZ = F16 ? 2 : 1;
  constexpr int KSTEPS = BK_BYTES / 32;
  constexpr int TCOLS = tmem_cols(TN);
  constexpr int PSTR = SWAP ? (BM + 4) : (TN + 4);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t *smem = (uint8_t *)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint8_t *sR = smem;
  uint8_t *sS = smem + STAGES * R_BYTES;
  uint8_t *sN = sS + STAGES * S_BYTES;
  uint64_t *bars = (uint64_t *)(sN + STAGES * NIB_BYTES);  // full[S], empty[S], conv[S], wfull[S], done
  uint32_t *tmem_slot = (uint32_t *)(bars + 4 * STAGES + 1);
  uint32_t *P = (uint32_t *)smem;
  uint8_t *sW = SWAP ? sR : sS;

  asm volatile("griddepcontrol.launch_dependents;");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t crank = cluster_ctarank();
  const uint32_t half = crank & 1u, leader_rank = crank & ~1u, peer_rank = crank ^ 1u;
  const bool leader = half == 0;
  const int r0 = (blockIdx.x >> 1) * (2 * BM), c0 = blockIdx.y * TN;  // pair tile origin
  const int rr = r0 + (int)half * BM, sr = c0 + (int)half * HS;        // this CTA's R rows / S rows
  const int SK = gridDim.z, ks = blockIdx.z;
  const int KB = (K * ESZ + BK_BYTES - 1) / BK_BYTES;
  const int kb0 = (int)((long long)KB * ks / SK), kb1 = (int)((long long)KB * (ks + 1) / SK);
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + STAGES), conv0 = smem_u32(bars + 2 * STAGES),
                 wfull0 = smem_u32(bars + 3 * STAGES), done = smem_u32(bars + 4 * STAGES);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full0 + 8 * s, 1);
      mbar_init(empty0 + 8 * s, 1);
      mbar_init(conv0 + 8 * s, 8);  // four converter warps in each CTA of the pair
      mbar_init(wfull0 + 8 * s, 1);
    }
    mbar_init(done, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mapR) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(&mapS) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TCOLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  cluster_sync();  // both CTAs' barriers and TMEM exist before any peer signal or MMA
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  // integer split-K: every split reduce-adds into C after split 0's pair has zeroed it, ordered by a
  // split-phase cluster barrier (see gemm_tc_kernel); the warps that arrive early complete that phase
  // before the final cluster barrier
  const bool tma_reduce = !F16 && SK > 1;
  const bool flagz = tma_reduce && tflag != nullptr;  // tile flags instead (each CTA's half its own flag)
  unsigned int *tf = flagz ? tflag + 2 * (blockIdx.y * gridDim.x + blockIdx.x) : nullptr;
  if (tma_reduce && !flagz && (warp < 2 || ks != 0)) cluster_arrive();

  auto load_w = [&](int s, int kb) {
    if constexpr (NIB) {
      tma_load_2d(smem_u32(sN + s * NIB_BYTES), SWAP ? &mapR : &mapS, kb * 64, SWAP ? rr : sr, wfull0 + 8 * s);
    } else {
      const int x = kb * (BK_BYTES / ESZ);
      if (SWAP) tma_load_2d_pair(smem_u32(sR + s * R_BYTES), &mapR, x, rr, mapa_u32(full0 + 8 * s, leader_rank));
      else tma_load_2d_pair(smem_u32(sS + s * S_BYTES), &mapS, x, sr, mapa_u32(full0 + 8 * s, leader_rank));
    }
  };
  auto load_a = [&](int s, int kb) {
    const int x = kb * (BK_BYTES / ESZ);
    if (SWAP) tma_load_2d_pair(smem_u32(sS + s * S_BYTES), &mapS, x, sr, mapa_u32(full0 + 8 * s, leader_rank));
    else tma_load_2d_pair(smem_u32(sR + s * R_BYTES), &mapR, x, rr, mapa_u32(full0 + 8 * s, leader_rank));
  };
  auto prefetch_a = [&](int kb) {
    const int x = kb * (BK_BYTES / ESZ);
    if (SWAP) tma_prefetch_2d(&mapS, x, sr);
    else tma_prefetch_2d(&mapR, x, rr);
  };
  auto expect = [&](int s) {
    if (leader) mbar_expect_tx(full0 + 8 * s, FULL_TX);
    if (NIB) mbar_expect_tx(wfull0 + 8 * s, NIB_BYTES);
  };

  if (warp == 0) {
    if (lane == 0) {
      const int ring = (kb1 - kb0) < STAGES ? (kb1 - kb0) : STAGES;  // (as in gemm_tc_kernel)
      const int pre = prew < ring ? prew : ring;
      for (int i = 0; i < pre; i++) {
        expect(i);
        load_w(i, kb0 + i);
      }
      if (SWAP ? (blockIdx.x & 15) < 2 : blockIdx.y == 0)  // L2 hint before the wait (see gemm_tc_kernel)
        for (int i = 0; i < ring; i++) prefetch_a(kb0 + i);
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int i = 0; i < pre; i++) load_a(i, kb0 + i);
      for (int i = pre; i < ring; i++) {
        expect(i);
        load_a(i, kb0 + i);
        load_w(i, kb0 + i);
      }
      for (int kb = kb0 + ring; kb < kb1; kb++) {
        const int i = kb - kb0, s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(empty0 + 8 * s, ph ^ 1u)) break;
        expect(s);
        load_w(s, kb);
        load_a(s, kb);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      constexpr uint32_t id = idesc_pair<F16>(TN);
      for (int kb = kb0; kb < kb1; kb++) {
        const int i = kb - kb0, s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        if (!mbar_wait(full0 + 8 * s, ph)) break;
        if (NIB && !mbar_wait_cluster(conv0 + 8 * s, ph)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t rd = sw128_desc(smem_u32(sR + s * R_BYTES));
        const uint64_t sd = sw128_desc(smem_u32(sS + s * S_BYTES));
#pragma unroll
        for (int k = 0; k < KSTEPS; k++)
          umma_pair<F16>(tmem, rd + 2 * k, sd + 2 * k, id, (kb > kb0 || k > 0) ? 1u : 0u);
        umma_commit_pair(empty0 + 8 * s);
        umma_commit_pair(mapa_u32(empty0 + 8 * s, peer_rank));
      }
      umma_commit_pair(done);
      umma_commit_pair(mapa_u32(done, peer_rank));
    }
  } else {
    const int ct = threadIdx.x - 64;
    if (tma_reduce && ks == 0) {  // this CTA's 128-row half of the tile, zeroed after the previous grid
      asm volatile("griddepcontrol.wait;" ::: "memory");
      const int rows = SWAP ? min(TN, M - c0) : min(BM, M - rr);
      const int cols = SWAP ? min(BM, N - rr) : min(TN, N - c0);
      const int m0 = SWAP ? c0 : rr, n0 = SWAP ? rr : c0, vpr = cols / 4;
      uint32_t *Cz = (uint32_t *)Cout;
      for (int t = ct; t < rows * vpr; t += 128)
        *reinterpret_cast<uint4 *>(Cz + (size_t)(m0 + t / vpr) * N + n0 + 4 * (t % vpr)) = make_uint4(0, 0, 0, 0);
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncwarp();
      if (flagz) {
        epi_bar_sync();
        if (ct == 0) tile_flag_set(tf);
      } else {
        cluster_arrive();
      }
    }
    if (!NIB && flagz && ks != 0) tile_flag_pass(tf, ct);  // while the accumulator fills (see gemm_tc_kernel)
    if constexpr (NIB) {
      bool cok = true;
      for (int kb = kb0; kb < kb1 && cok; kb++) {
        const int i = kb - kb0, s = i % STAGES;
        const uint32_t ph = (uint32_t)(i / STAGES) & 1u;
        cok = mbar_wait(wfull0 + 8 * s, ph);
        if (!cok) break;
        const uint8_t *src = sN + s * NIB_BYTES;
        uint8_t *dst = sW + s * (SWAP ? R_BYTES : S_BYTES);
        expand_stage<FMT, WROWS>(src, dst, ct, tb);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(mapa_u32(conv0 + 8 * s, leader_rank));
      }
    }
    if (tma_reduce) {
      if (flagz) {
        if (NIB && ks != 0) tile_flag_pass(tf, ct);
      } else {
        __syncwarp();
        cluster_wait();
      }
      asm volatile("fence.proxy.async.global;" ::: "memory");
    }
    const int sub = warp & 3;
    const bool ok = mbar_wait(done, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (ok) {
      if (F16 && SK > 1) {
        drain_rows<SWAP, TN, PSTR>(tmem + ((uint32_t)(sub * 32) << 16), lane, true, P, sub * 32 + lane,
                                   (uint32_t *)smem + sub * 32 * kStgStride, (uint32_t *)Cout, M, N, rr + sub * 32,
                                   c0);
      } else if constexpr (SWAP) {
        const uint32_t sbox = smem_u32(smem) + (uint32_t)(sub * TN * 128);
        drain_cols_tma<TN>(tmem + ((uint32_t)(sub * 32) << 16), lane, sbox);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0 && rr + sub * 32 < N && c0 < M) {
          if (tma_reduce) tma_reduce_add_2d(&mapC, rr + sub * 32, c0, sbox);
          else tma_store_2d(&mapC, rr + sub * 32, c0, sbox);
          bulk_commit();
        }
      } else {
        drain_rows_tma<TN>(tmem + ((uint32_t)(sub * 32) << 16), lane, smem_u32(smem) + (uint32_t)(sub * 4096), &mapC,
                           c0, rr + sub * 32, M, N, tma_reduce);
      }
    }
    if (flagz && ct == 0) tile_flag_count(tf, SK);
    if (lane == 0) bulk_wait_read();
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncwarp();
  if (tma_reduce && !flagz && warp < 2) cluster_wait();  // the early arrivals' phase, before the final barrier
  if (F16 && SK > 1) {
    cluster_sync();
    // this CTA's slice of its half-tile: (output row, 4-column vector) items in C's row-major order,
    // summed over the partials of cluster ranks half + 2q
    const int out_rows = SWAP ? min(TN, M - c0) : min(BM, M - rr);
    const int out_cols = SWAP ? min(BM, N - rr) : min(TN, N - c0);
    const int vpr = out_cols / 4;
    const int items = out_rows > 0 && out_cols > 0 ? out_rows * vpr : 0;
    reduce_split_any<F16>(SK, smem_u32(P), PSTR, ks * 192 + (int)threadIdx.x, SK * 192, items, vpr, half, 2u,
                          (uint32_t *)Cout, N, SWAP ? c0 : rr, SWAP ? rr : c0);
  }
  cluster_sync();  // the pair (and every split-K partial) is finished before TMEM and shared memory go
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TCOLS));
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

// 2-D map over a row-major [rows][row_bytes] byte matrix (element = esz bytes) with a box of
// box_rows x box_bytes; 128-byte swizzle for MMA operand tiles, none for the nibble staging tiles.
bool make_map(CUtensorMap *map, const void *base, int rows, size_t row_bytes, int esz, int box_rows,
              int box_bytes, bool swizzle,
              CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_UINT8) {
  auto fn = encode_fn();
  if (!fn) return false;
  if (esz == 2) dtype = CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / esz), (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)(box_bytes / esz), (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, dtype, 2, const_cast<void *>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// The output map: C [M][N] of 4-byte elements (s32 sums, or f32 for fp16 runs), boxes of 32 columns by
// 32 rows with the 128-byte swizzle for row tiles, or by TN rows unswizzled for swapped tiles.
bool make_c_map(CUtensorMap *map, void *C, int M, int N, bool f32, bool swap, int tn) {
  return make_map(map, C, M, (size_t)N * 4, 4, swap ? tn : 32, 128, !swap,
                  f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_INT32);
}


template <int FMT, bool SWAP, int TN, int STAGES, int NA = 1>
cudaError_t launch_tc(const RunArgs &a, int sk, cudaStream_t s, bool pdl) {
  constexpr bool NIB = FMT == FMT_U4 || FMT == FMT_NF4;
  constexpr int ESZ = FMT == FMT_F16 ? 2 : 1;
  constexpr int TM = BM * NA;
  constexpr int WROWS = SWAP ? TM : TN;
  CUtensorMap mR, mS;
  const size_t a_row = (size_t)a.K * ESZ, w_row = fmt_row_bytes(FMT, a.K);
  // the weight operand: its MMA tile (int8/f16, swizzled) or its nibble staging tile (64 B per row)
  const bool okW = NIB ? make_map(SWAP ? &mR : &mS, a.W, a.N, w_row, 1, WROWS, 64, false)
                       : make_map(SWAP ? &mR : &mS, a.W, a.N, w_row, ESZ, WROWS, BK_BYTES, true);
  const bool okA = make_map(SWAP ? &mS : &mR, a.A, a.M, a_row, ESZ, SWAP ? TN : TM, BK_BYTES, true);
  CUtensorMap mC;
  const bool okC = make_c_map(&mC, a.C, a.M, a.N, FMT == FMT_F16, SWAP, TN);
  if (!okW || !okA || !okC) return cudaErrorInvalidValue;
  constexpr size_t ring = (size_t)STAGES * ((TM + TN) * BK_BYTES + (NIB ? WROWS * 64 : 0));
  constexpr size_t part = (size_t)(SWAP ? TN * (TM + 4) : TM * (TN + 4)) * 4;
  static_assert(part <= ring, "partial tile must fit in the stage ring");
  constexpr size_t staging = SWAP ? (size_t)4 * TN * 128 : (size_t)TM * TN * 4;
  static_assert(staging <= ring, "the output staging boxes must fit in the stage ring");
  constexpr size_t smem = 1024 + ring + (3 * STAGES + 1) * 8 + 16;
  static_assert(smem <= 232448, "shared memory budget");
  auto kern = gemm_tc_kernel<FMT, SWAP, TN, STAGES, NA>;
  {
    const cudaError_t e = smem_attr((const void *)kern, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const Nf4Tables tb = nf4_tables();
  const int rowsR = SWAP ? a.N : a.M, rowsS = SWAP ? a.M : a.N;
  const int gx = (rowsR + TM - 1) / TM, gy = (rowsS + TN - 1) / TN;
  // integer split-K with the context's tile flags: the splits need not share a cluster. Row tiles only:
  // decode-sized (swapped) grids split up to 8 ways into short K ranges, where a cluster barrier was
  // measured faster (int8 M = 8: 2048x2048 2.98 against 3.6 us, 6144x2048 4.65 against 5.2) -- except
  // splits of more than 8, which no cluster holds
  if (sk > 8 && (FMT == FMT_F16 || !a.tflag || gx * gy > kTcFlagTiles)) sk = 8;
  const bool flagz = (!SWAP || sk > 8) && FMT != FMT_F16 && sk > 1 && a.tflag && gx * gy <= kTcFlagTiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gx, gy, sk);
  cfg.blockDim = dim3(tc_threads<FMT, SWAP>());
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = 1;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = flagz ? 1 : sk;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  // weight stages requested before the dependency wait: the whole ring, except the 8-deep ring of the
  // 64-wide row tiles, where two and then activations first measured faster (6144x2048xM128 8.0 -> 7.5 us;
  // the other prefill shapes within 1 %, decode-sized grids slower with fewer)
  const int prew = a.tune && a.tune->tc_pre > 0 ? a.tune->tc_pre : (!SWAP && STAGES >= 8) ? 2 : STAGES;
  return cudaLaunchKernelEx(&cfg, kern, mR, mS, mC, a.C, a.M, a.N, a.K, tb, flagz ? a.tflag : (unsigned int *)nullptr,
                            prew);
}

// CTA-pair launch: grid x = 2 CTAs per 256 R rows, y = S tiles of TN, z = split-K; cluster (2, 1, sk).
template <int FMT, bool SWAP, int TN, int STAGES>
cudaError_t launch_tc_pair(const RunArgs &a, int sk, cudaStream_t s, bool pdl) {
  constexpr bool NIB = FMT == FMT_U4 || FMT == FMT_NF4;
  constexpr int ESZ = FMT == FMT_F16 ? 2 : 1;
  constexpr int HS = TN / 2;
  constexpr int WROWS = SWAP ? BM : HS;
  static_assert(TN % 32 == 0 && TN >= 64 && TN <= 256, "pair MMA N");
  if (sk < 1 || sk > 4) return cudaErrorInvalidValue;
  CUtensorMap mR, mS;
  const size_t a_row = (size_t)a.K * ESZ, w_row = fmt_row_bytes(FMT, a.K);
  const bool okW = NIB ? make_map(SWAP ? &mR : &mS, a.W, a.N, w_row, 1, WROWS, 64, false)
                       : make_map(SWAP ? &mR : &mS, a.W, a.N, w_row, ESZ, WROWS, BK_BYTES, true);
  const bool okA = make_map(SWAP ? &mS : &mR, a.A, a.M, a_row, ESZ, SWAP ? HS : BM, BK_BYTES, true);
  CUtensorMap mC;
  const bool okC = make_c_map(&mC, a.C, a.M, a.N, FMT == FMT_F16, SWAP, TN);
  if (!okW || !okA || !okC) return cudaErrorInvalidValue;
  constexpr size_t ring = (size_t)STAGES * ((BM + HS) * BK_BYTES + (NIB ? WROWS * 64 : 0));
  constexpr size_t part = (size_t)(SWAP ? TN * (BM + 4) : BM * (TN + 4)) * 4;
  static_assert(part <= ring, "partial tile must fit in the stage ring");
  constexpr size_t staging = SWAP ? (size_t)4 * TN * 128 : (size_t)BM * TN * 4;
  static_assert(staging <= ring, "the output staging boxes must fit in the stage ring");
  constexpr size_t smem = 1024 + ring + (4 * STAGES + 1) * 8 + 16;
  static_assert(smem <= 232448, "shared memory budget");
  auto kern = gemm_tc_pair_kernel<FMT, SWAP, TN, STAGES>;
  {
    const cudaError_t e = smem_attr((const void *)kern, (int)smem);
    if (e != cudaSuccess) return e;
  }
  const Nf4Tables tb = nf4_tables();
  const int rowsR = SWAP ? a.N : a.M, rowsS = SWAP ? a.M : a.N;
  const int gx = 2 * ((rowsR + 2 * BM - 1) / (2 * BM)), gy = (rowsS + TN - 1) / TN;
  const bool flagz = !SWAP && FMT != FMT_F16 && sk > 1 && a.tflag && gx * gy <= kTcFlagTiles;  // (as launch_tc)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(gx, gy, sk);
  cfg.blockDim = dim3(192);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  at[1].id = cudaLaunchAttributeClusterDimension;
  at[1].val.clusterDim.x = 2;
  at[1].val.clusterDim.y = 1;
  at[1].val.clusterDim.z = flagz ? 1 : sk;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kern, mR, mS, mC, a.C, a.M, a.N, a.K, tb, flagz ? a.tflag : (unsigned int *)nullptr,
                            a.tune && a.tune->tc_pre > 0 ? a.tune->tc_pre : STAGES);
}

struct TcCfg {
  bool swap;
  int tn, sk;
  int na = 1;         // 128-row accumulators per CTA along the R side
  int stages = 0;     // 0: the variant's default; 3: the 96 KB ring of the 128 x 128 tile
  bool pair = false;  // CTA-pair (cta_group::2) tile of 256 x tn
};

// Tile and split choice. Swapped operands with the narrowest N-tile covering M for M <= 64 (weight
// streaming; K split over a cluster up to 8 ways while the grid stays within ~320 CTAs, two per SM).
// For larger M, measured on B200 over configs of K in {2048, 6144}, N in {2048, 6144, 12288},
// M in {128, 256, 512} with a per-phase timeline of the kernel: a CTA streams its operands at ~115 GB/s
// (the TMA's rate per SM, from L2 or HBM alike) and writes its C tile at ~60 GB/s, and every launch
// carries ~2-3 us of fixed latency (first data after the dependency wait, the gap to the next launch).
// So the grid should cover the SMs once: 128-wide weight tiles, widened to 192 then 256 (int8 / f16)
// only while the grid would exceed one wave of 148 CTAs; nibble weights past one wave use CTA-pair tiles
// of 256 x 192 (the converter work per CTA halves); then split-K (integer partial tiles reduce-added by
// the TMA) as far as below.
TcCfg choose_tc(int fmt, int M, int K, int N, const Tuning &tu) {
  TcCfg c;
  const bool nib = fmt == FMT_U4 || fmt == FMT_NF4;
  const int KB = (K * (fmt == FMT_F16 ? 2 : 1) + BK_BYTES - 1) / BK_BYTES;
  c.swap = M <= 64;
  if (c.swap) {
    c.tn = M <= 16 ? 16 : M <= 32 ? 32 : 64;
    const int tiles = (N + BM - 1) / BM;
    c.sk = 1;
    while (tiles * c.sk * 2 <= 320 && c.sk * 2 <= 8 && c.sk * 2 <= KB) c.sk *= 2;
    // long int8 rows (K >= 6144): a 6-deep ring streams faster (6144x2048, M 8 / 16: 6.2 -> 5.6 us); for
    // shorter rows the default ring, with more CTAs resident for the next launch, is as fast or faster
    if (!nib && fmt != FMT_F16 && c.tn <= 32 && KB >= 48) c.stages = 6;
    // nibble weights whose unsplit grid already exceeds two CTAs per SM (wide N, M <= 16): the 2-stage
    // ring (up to four CTAs, so twice the converter warps, per SM) with a 2-way split measured fastest
    // (NF4 8192x57344xM8 80.6 -> 70.5 us, 8192x42752xM8 67.5 -> 56.5 us); on smaller grids it is slower
    if (nib && c.tn == 16 && tiles > 2 * 148 && KB >= 2) {
      c.stages = 2;
      c.sk = 2;
    }
    // narrow nibble weights with long rows (the 70B linears' column shards, configs[2]'s 6144x2048) stop
    // at 8 splits for the cluster; with the tile flags they split further while the grid stays within
    // 256 CTAs. NF4 M = 8: 8192x1024 6.3 -> 4.9 us (16), 28672x2048 19.9 -> 12.2 (16), 8192x2560 7.5 ->
    // 6.4 (12; 16 on 320 CTAs was slower), 6144x2048 6.2 -> 4.7; M = 32: 6144x2048 NF4 7.0 -> 5.1, uniform
    // 6.4 -> 4.8. (int8 weights measured slower past 8 splits.)
    if (nib && c.tn <= 32 && c.sk == 8 && KB >= 48 && tu.tc_flags)
      for (int s : {16, 12})
        if (tiles * s <= 256) {
          c.sk = s;
          break;
        }
  } else {
    const int mt = (M + BM - 1) / BM;
    auto tiles = [&](int tn) { return mt * ((N + tn - 1) / tn); };
    c.tn = 128;
    if (tiles(128) > 148) {
      if (nib) {
        c.pair = true;
        c.tn = ((M + 255) / 256) * ((N + 191) / 192) * 2 <= 148 ? 192 : 256;
      } else {
        c.tn = tiles(192) <= 148 ? 192 : 256;
      }
    }
    const int t = c.pair ? 2 * ((M + 255) / 256) * ((N + c.tn - 1) / c.tn) : tiles(c.tn);
    // split K as far as the grid stays one wave with room for cluster placement (132 of 148 SMs: clusters
    // of 3 or more do not pack every GPC), every split keeps at least 4 k-blocks, and the cluster stays
    // at most 6 CTAs (8-CTA clusters scheduled in two waves on these grids). Measured over the BASELINE
    // shapes: 2048x6144xM128 7.6 us at split 2 vs 8.6 unsplit and 12.7 at split 3 (144 CTAs);
    // 6144x2048xM128 7.4 us at 6 vs 8.0 at 4; 2048x2048xM512 7.7 at 2 vs 8.5 unsplit.
    c.sk = 1;
    for (int s : {2, 3, 4, 6})
      if (t * s <= 132 && KB / s >= 4 && (!c.pair || s <= 2)) c.sk = s;
    // int8 weights with the split-K tile flags (the splits then share no cluster, so any split and up to
    // one full wave of 148 CTAs): tile width and split from a cost model fitted to a sweep of the
    // BASELINE prefill shapes (M 128-512, K and N 2048 / 6144, widths 64-256, splits 1-6; mean error
    // 0.4 us): us = 4.17 + 0.0088 * operand KB per CTA + 0.0052 * C KB per CTA + 0.166 * MB of C that
    // all splits write. It trades the per-SM operand stream (narrower tiles re-read more of A and W)
    // against the int32 tile drain and the split partials the L2 adds up; every split keeps >= 5
    // k-blocks. Measured against the rule above: 6144x2048xM512 12.6 -> 11.6 us (192 wide, split 3),
    // 2048x2048xM128 6.6 -> 5.4 us (64 wide), 2048x6144xM128 7.9 -> 7.5 us (split 3, 144 CTAs).
    if (fmt == FMT_I8 && tu.tc_flags) {
      double best = 1e30;
      for (int tn : {64, 128, 192, 256})
        for (int s : {1, 2, 3, 4, 6}) {
          const long long ctas = (long long)tiles(tn) * s;
          if (ctas > 148 || (s > 1 && KB / s < 5)) continue;
          const double in_kb = (double)K / s * (128 + tn) / 1024.0, out_kb = 128.0 * tn * 4 / 1024.0;
          const double us = 4.17 + 0.0088 * in_kb + 0.0052 * out_kb + 0.166 * (double)ctas * out_kb / 1024.0;
          if (us < best) best = us, c.tn = tn, c.sk = s;
        }
    }
  }
  // tuning overrides (the context's ORKB_TC_* values): tile width, accumulators, ring depth, split
  if (!c.swap) {
    if (tu.tc_tn) c.tn = (!nib && (tu.tc_tn == 256 || tu.tc_tn == 192 || tu.tc_tn == 64)) ? tu.tc_tn : 128;
    if (tu.tc_na) c.na = tu.tc_na == 2 ? 2 : 1;
    if (c.na == 2) c.tn = 128;
  }
  if (tu.tc_stages) c.stages = tu.tc_stages;
  // tc_pair: 1 = CTA-pair tiles (swapped operands for M <= 256), 2 = pair with A on the 256-row side,
  // 3 = pair with the weight on the 256-row side (M <= 256)
  if (tu.tc_pair >= 1 && tu.tc_pair <= 3 && !(tu.tc_pair == 3 && M > 256)) {
    c.pair = true;
    c.na = 1;
    c.swap = tu.tc_pair == 3 || (tu.tc_pair == 1 && M <= 256);
    if (c.swap) c.tn = M <= 64 ? 64 : M <= 128 ? 128 : 256;
    else c.tn = (tu.tc_tn == 64 || tu.tc_tn == 128 || tu.tc_tn == 192) ? tu.tc_tn : 256;
    if (c.sk > 4) c.sk = 4;
  }
  if (tu.tc_sk >= 1 && tu.tc_sk <= (c.pair ? 4 : 16) && tu.tc_sk <= KB) c.sk = tu.tc_sk;
  return c;
}

template <int FMT>
cudaError_t dispatch(const RunArgs &a, const TcCfg &c, cudaStream_t s, bool pdl) {
  constexpr bool NIB = FMT == FMT_U4 || FMT == FMT_NF4;
  // swapped (decode-sized M) tiles keep the ring at 72-98 KB so two or three CTAs fit on an SM: the
  // next launch's CTAs then start streaming their weights while this one drains (programmatic launch)
  if (c.pair) {
    if (c.swap) {
      if (c.tn == 64) return launch_tc_pair<FMT, true, 64, 6>(a, c.sk, s, pdl);
      if (c.tn == 128) return launch_tc_pair<FMT, true, 128, NIB ? 5 : 6>(a, c.sk, s, pdl);
      return launch_tc_pair<FMT, true, 256, NIB ? 4 : 6>(a, c.sk, s, pdl);
    }
    if (c.tn == 64) return launch_tc_pair<FMT, false, 64, 8>(a, c.sk, s, pdl);
    if (c.tn == 128) return launch_tc_pair<FMT, false, 128, 6>(a, c.sk, s, pdl);
    if (c.tn == 192) return launch_tc_pair<FMT, false, 192, NIB ? 4 : 6>(a, c.sk, s, pdl);
    return launch_tc_pair<FMT, false, 256, NIB ? 4 : 6>(a, c.sk, s, pdl);
  }
  if (c.swap) {
    if constexpr (!NIB) {  // deeper rings (tuning override ORKB_TC_STAGES = 6 or 8)
      if (c.stages == 8) {
        if (c.tn == 16) return launch_tc<FMT, true, 16, 8>(a, c.sk, s, pdl);
        if (c.tn == 32) return launch_tc<FMT, true, 32, 8>(a, c.sk, s, pdl);
        return launch_tc<FMT, true, 64, 6>(a, c.sk, s, pdl);
      }
      if (c.stages == 6) {
        if (c.tn == 16) return launch_tc<FMT, true, 16, 6>(a, c.sk, s, pdl);
        if (c.tn == 32) return launch_tc<FMT, true, 32, 6>(a, c.sk, s, pdl);
        return launch_tc<FMT, true, 64, 5>(a, c.sk, s, pdl);
      }
    }
    if constexpr (NIB) {  // tuning override ORKB_TC_STAGES = 2: a 53-56 KB ring, up to four CTAs per SM
      if (c.stages == 2) {
        if (c.tn == 16) return launch_tc<FMT, true, 16, 2>(a, c.sk, s, pdl);
        if (c.tn == 32) return launch_tc<FMT, true, 32, 2>(a, c.sk, s, pdl);
      }
    }
    if (c.tn == 16) return launch_tc<FMT, true, 16, NIB ? 3 : 4>(a, c.sk, s, pdl);
    if (c.tn == 32) return launch_tc<FMT, true, 32, NIB ? 3 : 4>(a, c.sk, s, pdl);
    return launch_tc<FMT, true, 64, 3>(a, c.sk, s, pdl);
  }
  if (c.na == 2) return launch_tc<FMT, false, 128, NIB ? 3 : 4, 2>(a, c.sk, s, pdl);
  if constexpr (!NIB) {
    if (c.tn == 256) return launch_tc<FMT, false, 256, 4>(a, c.sk, s, pdl);
    if (c.tn == 192) return launch_tc<FMT, false, 192, 4>(a, c.sk, s, pdl);
    if (c.tn == 64) return launch_tc<FMT, false, 64, 8>(a, c.sk, s, pdl);
    if (c.stages == 3) return launch_tc<FMT, false, 128, 3>(a, c.sk, s, pdl);
  }
  return launch_tc<FMT, false, 128, NIB ? 4 : 6>(a, c.sk, s, pdl);
}

}  // namespace

bool gemm_tc_supports(int fmt, int M, int K, int N) {
  (void)K;
  if (fmt != FMT_I8 && fmt != FMT_F16 && fmt != FMT_U4 && fmt != FMT_NF4) return false;
  if (N % 16) return false;
  return M >= 1 && encode_fn() != nullptr;
}

cudaError_t launch_gemm_tc(const RunArgs &a, cudaStream_t s, bool pdl, int *launches) {
  if ((uintptr_t)a.A % 16 || (uintptr_t)a.W % 16 || (uintptr_t)a.C % 16) return cudaErrorMisalignedAddress;
  static const Tuning none;
  const TcCfg c = choose_tc(a.fmt, a.M, a.K, a.N, a.tune ? *a.tune : none);
  cudaError_t e;
  switch (a.fmt) {
    case FMT_I8: e = dispatch<FMT_I8>(a, c, s, pdl); break;
    case FMT_F16: e = dispatch<FMT_F16>(a, c, s, pdl); break;
    case FMT_U4: e = dispatch<FMT_U4>(a, c, s, pdl); break;
    case FMT_NF4: e = dispatch<FMT_NF4>(a, c, s, pdl); break;
    default: return cudaErrorNotSupported;
  }
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

ORKB_ERR_WORD_SETTER(tc_set_err_word)

}  // namespace orkb

extern "C" int ork_b200_tc_choice(int fmt, int M, int K, int N, int *out) {
  if (!out || fmt < orkb::FMT_F16 || fmt > orkb::FMT_NF4 || M < 1 || K < 1 || N < 1) return -1;
  const orkb::TcCfg c = orkb::choose_tc(fmt, M, K, N, orkb::tuning_from_env());
  out[0] = c.swap ? 1 : 0;
  out[1] = c.tn;
  out[2] = c.sk;
  out[3] = c.stages;
  out[4] = c.pair ? 1 : 0;
  return 0;
}

// ork_internal.h -- shared definitions of the B200 resident-weight matmul engine (not installed).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace orkb {

// Resident weight formats. Every format keeps the weight K-major, i.e. as B^T with one output channel
// per row, so a channel's K values are contiguous in HBM:
//   FMT_F16 : [N][K] IEEE binary16
//   FMT_I8  : [N][K] int8 codes
//   FMT_U4  : [N][K/2] bytes, two's-complement int4 codes, low nibble = even k (the O4N1 nibble layout)
//   FMT_NF4 : [N][K/2] bytes, NF4 codebook indices 0..15, low nibble = even k (the O4N1 nibble layout)
enum Fmt { FMT_F16 = 0, FMT_I8 = 1, FMT_U4 = 2, FMT_NF4 = 3 };

// Device ordinals the per-device tables (error words, no-allocation scratch addresses) cover.
constexpr int kMaxDevices = 64;

// Which public run function a weight belongs to (ork-driver src/npu/internal.h DT_* values).
enum ApiDtype { DT_F16 = 0, DT_I8 = 1, DT_I4 = 2 };

inline size_t fmt_row_bytes(int fmt, int K) {
  return fmt == FMT_F16 ? (size_t)K * 2 : fmt == FMT_I8 ? (size_t)K : (size_t)K / 2;
}

// The NF4 int8 lookup table lut[i] = rint(level[i]*127) (ork-driver src/npu/i4/pack.c:128-131 with the
// levels of src/npu.c:888-892), as the kernels use it: two 8-byte tables whose entries are all >= 0,
// negneg = -lut[0..7] and pos = lut[8..15].
extern const int8_t kNf4Lut[16];

// Tuning overrides of the kernel choice, from the ORKB_* environment variables. A context takes them
// once, when it is created (or again on ork_b200_reload_tuning), never per launch; 0 / -1 leave the
// router's own choice:
//   tc_tn ORKB_TC_TN (128/192/256), tc_na ORKB_TC_NA (1/2), tc_stages ORKB_TC_STAGES, tc_pair ORKB_TC_PAIR
//   (1..3), tc_sk ORKB_TC_SK (1..8), tc_flags ORKB_TC_FLAGS (0: split-K zeroing ordered through a
//   cluster barrier instead of the tile flags), tc_pre ORKB_TC_PRE (weight stages requested before the
//   dependency wait; default the whole ring); gemv_kind ORKB_GEMV_KIND (0 staged / 1 direct), gemv_cpw
//   ORKB_GEMV_CPW (1/2/4), gemv_tr ORKB_GEMV_TR (8/16/32), gemv_nw ORKB_GEMV_NW (4/8/16 warps);
//   layer_fused ORKB_LAYER_FUSED (0 multi-launch).
struct Tuning {
  int tc_tn = 0, tc_na = 0, tc_stages = 0, tc_pair = 0, tc_sk = 0, tc_flags = 1, tc_pre = 0;
  int pipe = 1;  // ORKB_PIPE: 0 = large host-buffer runs in one piece instead of row blocks; 2..8 = most blocks
  int gemv_kind = -1, gemv_cpw = 0, gemv_tr = 0, gemv_nw = 0;
  int layer_fused = -1;
};
Tuning tuning_from_env();

// ---- kernel launchers (gemv.cu, gemm_sm100.cu) --------------------------------------------------
struct RunArgs {
  const void *W;   // resident weight
  const void *A;   // device activations [M][K] (int8 or fp16), 16-byte aligned rows
  void *C;         // device output [M][N] (int32 or fp32)
  int M, K, N;
  int fmt;
  const Tuning *tune = nullptr;  // the context's tuning overrides (nullptr: none)
  // The context's split-K tile flags for the tensor-core kernel (kTcFlagTiles x 2 words, zero between
  // launches), or nullptr: split-K then orders its zeroing through a cluster barrier instead.
  unsigned int *tflag = nullptr;
};
constexpr int kTcFlagTiles = 16384;

// Decode path: M <= 8 per launch (the launcher loops over row blocks of 8 for larger M). Two kernels:
// staged (a CTA copies 8 whole weight rows into shared memory) and direct-load (a warp streams its rows
// through registers); the direct one has no row-size limit, so every K is supported.
cudaError_t launch_gemv(const RunArgs &a, cudaStream_t s, bool pdl, int *launches);
inline bool gemv_supports(int fmt, int K) { return K > 0 && fmt >= FMT_F16 && fmt <= FMT_NF4; }
unsigned int gemv_error_flag(bool reset);
unsigned int layer_error_flag(bool reset);  // layer.cu: a position outside the caches
unsigned int peer_error_flag(bool reset);   // peers.cu: a peer wait expired
// Raise a kernel's dynamic shared-memory limit on the current device, once per (kernel, device): the
// attribute belongs to the device's context, so a process driving several GPUs needs it on each.
cudaError_t smem_attr(const void *kernel, int bytes);
// Point each module's kernels at the device's error word (errword.cuh); called once per device.
cudaError_t gemv_set_err_word(unsigned int *p);
cudaError_t tc_set_err_word(unsigned int *p);
cudaError_t layer_set_err_word(unsigned int *p);
cudaError_t fused_set_err_word(unsigned int *p);
cudaError_t peer_set_err_word(unsigned int *p);

// Grouped (per-K-group scaled) matmul, ork-driver src/npu/core/buf.c:501-520: C[m][n] fp32 = sum over
// groups g, ascending, of ((float)P_g[m][n] * aScale[m*Sk+g]) * bScale[g*N+n], P_g the exact int32 dot
// over the group's G columns; Sk = K/G. Weight formats FMT_I8 (G % 16 == 0), FMT_U4 / FMT_NF4
// (G % 32 == 0). Device pointers; M any (launched 8 rows at a time).
struct GroupedArgs {
  const void *W;
  const void *A;       // [M][K] int8
  const float *aS;     // [M][K/G]
  const float *bS;     // [K/G][N]
  float *C;            // [M][N]
  int M, K, N, fmt, G;
};
cudaError_t launch_gemv_grouped(const GroupedArgs &a, cudaStream_t s, bool pdl, int *launches);

// Batched decode: independent matmuls of one weight format in one launch of the staged decode kernel
// (the chain / MoE entry points); each task M <= 8 with rows that fit the staged kernel
// (batched_supports). C of task t is written at a row stride of cstride elements.
// Output stage of an int8-compute matmul (the reference's fused requant outputs, include/ork/run.h:48-108):
// OUT_I32 the raw int32 sums; OUT_I8 / OUT_I16 clamp(rne(acc * mult / 2^shift)) to int8 / int16;
// OUT_EWMUL clamp_i8(rne(acc * G * mult / 2^shift)) with G int8 laid out like C. rne = round half to even.
enum { OUT_I32 = 0, OUT_I8 = 1, OUT_I16 = 2, OUT_EWMUL = 3 };
// Column-sharded runs with the gather over peer memory (peers.cu).
constexpr int kMaxPeers = 8;
struct PeerTable {                 // device memory, written once when the table is created
  int n, rank, ldc, col0, ctas;    // ranks, this rank, C row stride, first column, shard columns
  int32_t *C[kMaxPeers];           // every rank's C [M][ldc], mapped in this process
  unsigned int *flag[kMaxPeers];   // every rank's signal counts [kMaxPeers] (index: signalling rank)
  unsigned int *waited;            // this rank's count of completed waits (private)
  unsigned int *done;              // CTAs of the current run finished (private, left at zero)
  // tagged-word gather (optional): every rank's landing buffer [land_rows][ldc] of 8-byte words (value
  // in the low half, the run's tag in the high half), this rank's count of tagged runs, and the CTAs of
  // the current tagged run finished (private, left at zero)
  uint64_t *land[kMaxPeers];
  int land_rows;
  unsigned int *runs, *ldone;
};
struct OutStage {
  int mode, mult, shift;
  const int8_t *G;
};
struct ChainTask {
  const void *W;
  const void *A;
  void *C;
  int M, K, N, cstride, fmt;
  OutStage os;  // zero: raw int32 C
};
bool batched_supports(int fmt, int M, int K);
// Elementwise output stages over n values (outstage.cu): requant of int32 sums, and the int8 x int8
// element-wise multiply of ork_i8_npu_ewmul.
cudaError_t launch_requant(const int32_t *C, size_t n, const OutStage &os, void *out, cudaStream_t s);
cudaError_t launch_ewmul_i8(const int8_t *a, const int8_t *b, size_t n, int mult, int shift, int8_t *out,
                            cudaStream_t s);

cudaError_t launch_gemv_batched(const ChainTask *t, int n, cudaStream_t s, bool pdl, int *launches);
bool grouped_supports(int fmt, int K, int G);

// Tensor-core path (tcgen05). Returns cudaErrorNotSupported when the shape/format has no TC kernel.
cudaError_t launch_gemm_tc(const RunArgs &a, cudaStream_t s, bool pdl, int *launches);
bool gemm_tc_supports(int fmt, int M, int K, int N);
// Sticky device flag a tensor-core kernel sets when one of its bounded mbarrier waits expired (the kernel
// then exits without a result). Read after a synchronisation; reset clears it.
unsigned int tc_error_flag(bool reset);

// Persistent decode layers (layer_fused.cu): one cooperative launch of one CTA per SM runs nl consecutive
// ork_i8_mm_layer steps (the residual stream passing from layer to layer on the device). The caller
// fills everything above `slot`; launch_layer_fused plans the shared memory (fused_plan: false when the
// layer's rows or activations do not fit it) and launches.
struct FusedLayerW {  // one layer's pointers (a table in device memory)
  const uint8_t *W[7];  // q, k, v, o, gate, up, down: resident rows of one int8-compute format
  const float *attn_norm, *q_norm, *k_norm, *ffn_norm;
  float *Kc, *Vc;       // caches [Hkv][hstride][dk]
};
struct FusedArgs {
  const FusedLayerW *lw;  // [nl] in device memory, or null for one layer described by lw0
  FusedLayerW lw0;
  int nl;
  int ext;                // append the token's k / v into the caches at slot nkv
  const float *x;         // the first layer's input
  float *x_out;           // the last layer's output
  int D, H, Hkv, dk, F, nkv, pos, hstride;
  const int *dpos;
  float scale, base;
  // values exchanged between CTAs: 64-bit words, the value's bits in the low half and the layer's tag
  // in the high half, so a reader can tell fresh from stale words without a fence
  uint64_t *q, *k, *v, *o;   // projections [H*dk], [Hkv*dk], [Hkv*dk], [D] (int32)
  uint64_t *pm, *pz, *po;    // attention chunk partials [H][Sg], [H][Sg], [H][Sg][dk] (float)
  uint64_t *ao, *amax;       // merged attention output [H][dk] and max |.| per head (float)
  uint64_t *h, *hmax;        // SwiGLU row [F] and max |h| per CTA [grid] (float)
  uint64_t *xl;              // the residual stream between layers [D] (float)
  unsigned int *epoch;       // tag of the last layer run (advanced by the last CTA to finish)
  unsigned int *sync;        // arrival counts [5]: heads merged, CTAs past o, past SwiGLU, finished,
                             // past the residual (all zeroed by the last CTA to finish)
  int Sg, kpc;               // attention chunks per head, most keys per chunk
  uint32_t slot;             // -- planned: ring slot bytes, slots, shared-memory layout
  int nslots;
  uint32_t off_a8, off_x, off_y, off_loc, smem;
};
int fused_grid(int device);                  // CTAs of the persistent launch: the device's SM count
int fused_splits(int H, int maxk, int G);    // attention chunks per head
int fused_kpc(int maxk, int Sg);             // most keys per chunk (a multiple of 32)
bool fused_plan(FusedArgs *a, int fmt, int G);
cudaError_t launch_layer_fused(const FusedArgs &a, int fmt, int G, cudaStream_t s);
unsigned int fused_error_flag(bool reset);

}  // namespace orkb

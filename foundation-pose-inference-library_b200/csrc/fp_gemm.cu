// Persistent tcgen05 implicit-GEMM kernel (sm_100a) for RefineNet / ScoreNet.
//
// One CTA per SM walks output tiles of 128 (or, for layers of at most 128
// output channels, 256) rows x BN channels; layers with 256-channel tiles run
// on CTA pairs instead (gemmPairKernel below) when their rows fill the GPU.
// Warp roles:
//   warp 0     producer: per 64-channel chunk, one bulk copy per channel plane
//              brings a window of 128 + span rows of the activation into shared
//              memory (reused by every tap of the convolution); per 64-wide K
//              stage a TMA tile load brings the weights (128B swizzle).
//   warp 1     MMA issuer + TMEM owner: tcgen05.mma kind::f16 (kind::tf32
//              for fp32), M=128, N=BN, K=16, fp32 accumulators in TMEM, two
//              accumulator buffers so the epilogue of tile i overlaps the MMAs
//              of tile i+1. The whole warp runs the issue loop, so descriptors
//              and loop state stay warp-uniform, and an elected lane issues
//              each instruction: the issue rate, not the tensor core, bounds
//              the narrow (N <= 128) layers, and a single-lane loop issued
//              measurably slower.
//   warps 2-9  epilogue, two warps per TMEM lane quarter (each converts half
//              of the BN columns, or with 256-row tiles one 128-row half):
//              tcgen05.ld rows of the accumulator, bias /
//              residual / positional embedding / ReLU, bf16|fp16 stores into
//              the KP8 destination layout chosen by the layer (see include/fpk.h).
// The activation window uses the no-swizzle K-major core-matrix layout
// [plane][row][16 B]; shifting a convolution tap by one row is a 16-byte move of
// the descriptor start address, so all taps read the same staged window.
// Every mbarrier wait is bounded: on timeout the kernel records an error code
// in desc.error_flag and all roles drain and exit.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <mutex>
#include <string>
#include <type_traits>
#include <unordered_map>

#include "fp_launch.hpp"
#include "fp_net_kernels.cuh"
#include "fp_profile.hpp"
#include "fp_tc.cuh"
#include "fpk.h"

namespace fpb {

int fail(const std::string& msg);
int checkLaunch(const char* what);

namespace gemm {

using namespace fpb::tc;

constexpr int kEpilogueWarps = 8;  // two per TMEM lane quarter, each takes half the columns
constexpr int kThreads = 64 + 32 * kEpilogueWarps;
constexpr int kBlockM = 128;
constexpr int kStageBytes = 128;  // K bytes per weight stage: 64 fp16/bf16 or 32 fp32 elements
constexpr int kMaxASlots = 8;
constexpr int kMaxBStages = 16;
constexpr int kMaxStagesPerChunk = FPK_GEMM_MAX_TAPS;  // 64-channel chunks: one stage per tap
constexpr size_t kSmemBytes = 220 * 1024;  // dynamic shared memory per CTA
constexpr size_t kOutStageBytes = 8 * 2 * 2048;  // staged output chunks: 8 epilogue warps x 2 x [4 planes][32 rows][16 B]

struct Smem {
  uint64_t a_full[kMaxASlots], a_empty[kMaxASlots];
  uint64_t b_full[kMaxBStages], b_empty[kMaxBStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  uint32_t pad;
  // Per stage within a channel chunk: the four K=16 steps' A descriptor start
  // offsets (16-byte units, relative to the window slot), packed 2 x u16 per word.
  uint2 a_off[kMaxStagesPerChunk];
};

// Element type traits. Every K step of the MMA reads 32 bytes of each row:
// K=16 for fp16/bf16 (kind::f16), K=8 for fp32 read as TF32 (kind::tf32).
// A 16-byte activation record holds 8 (16-bit) or 4 (fp32) channels.
template <typename T>
struct Elem {
  static constexpr int kBytes = sizeof(T);
  static constexpr int kPerRecord = 16 / kBytes;          // channels per 16-byte record
  static constexpr int kPerStage = kStageBytes / kBytes;  // K elements per weight stage
  static constexpr bool kTf32 = std::is_same<T, float>::value;
  // Instruction descriptor: fp32 accumulate, A/B K-major, A/B format F16=0 /
  // BF16=1 / TF32=2.
  static constexpr uint32_t fmt() { return kTf32 ? 2u : (std::is_same<T, __nv_bfloat16>::value ? 1u : 0u); }
  static constexpr uint32_t instrDesc(int bn, int m) {
    return (1u << 4) | (fmt() << 7) | (fmt() << 10) | (static_cast<uint32_t>(bn >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
  }
};

template <typename T>
__device__ __forceinline__ void mmaTElect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  if constexpr (Elem<T>::kTf32) {
    tcMmaTf32Elect(d_tmem, a_desc, b_desc, idesc, accumulate);
  } else {
    tcMmaElect(d_tmem, a_desc, b_desc, idesc, accumulate);
  }
}

struct Plan {
  int cw;            // channels per chunk (32 or 64)
  int planes;        // planes per chunk = cw / 8
  int n_chunks;      // cin / cw
  int stages_per_chunk;
  int min_off, win_rows;
  int a_slots;       // activation windows in flight (2..kMaxASlots)
  int b_stages;
  int m_tiles, n_tiles;
  uint32_t a_win_bytes;  // per slot
  uint32_t b_stage_bytes;
  uint32_t a_slot_bytes;  // CTA-pair kernel: window slot stride (1024-byte aligned)
  uint32_t a_plane_pitch;  // CTA-pair kernel: bytes between channel planes of a window (128-byte aligned)
  int k_splits;            // single-CTA kernel: CTAs sharing one output tile's K range (1 = no split)
  int withhold_loads;      // failure-injection test: the producer issues no loads (see fpk_gemm_test_withhold_loads)
  int tma_store;           // CTA-pair kernel, dense 16-bit outputs: epilogue stages 32-column chunks, TMA stores them
  uint32_t stage_off;      // offset of the staging area (8 warps x 2 x 2 KB) from the aligned dynamic smem base
};

template <typename T>
__device__ __forceinline__ uint4 pack8(const float* v);
template <>
__device__ __forceinline__ uint4 pack8<__nv_bfloat16>(const float* v) {
  uint4 o;
  __nv_bfloat162 h0 = __floats2bfloat162_rn(v[0], v[1]);
  __nv_bfloat162 h1 = __floats2bfloat162_rn(v[2], v[3]);
  __nv_bfloat162 h2 = __floats2bfloat162_rn(v[4], v[5]);
  __nv_bfloat162 h3 = __floats2bfloat162_rn(v[6], v[7]);
  o.x = *reinterpret_cast<uint32_t*>(&h0);
  o.y = *reinterpret_cast<uint32_t*>(&h1);
  o.z = *reinterpret_cast<uint32_t*>(&h2);
  o.w = *reinterpret_cast<uint32_t*>(&h3);
  return o;
}
template <>
__device__ __forceinline__ uint4 pack8<__half>(const float* v) {
  uint4 o;
  __half2 h0 = __floats2half2_rn(v[0], v[1]);
  __half2 h1 = __floats2half2_rn(v[2], v[3]);
  __half2 h2 = __floats2half2_rn(v[4], v[5]);
  __half2 h3 = __floats2half2_rn(v[6], v[7]);
  o.x = *reinterpret_cast<uint32_t*>(&h0);
  o.y = *reinterpret_cast<uint32_t*>(&h1);
  o.z = *reinterpret_cast<uint32_t*>(&h2);
  o.w = *reinterpret_cast<uint32_t*>(&h3);
  return o;
}

template <typename T>
__device__ __forceinline__ void unpack8(uint4 u, float* v);
template <>
__device__ __forceinline__ void unpack8<__nv_bfloat16>(uint4 u, float* v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void unpack8<__half>(uint4 u, float* v) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

// Eight consecutive channels starting at channel c (a multiple of 8) of row
// `row` in a planar activation: one 16-byte record for 16-bit types, two
// (channels c..c+3 and c+4..c+7 in consecutive planes) for fp32.
template <typename T>
__device__ __forceinline__ void loadRec8(const unsigned char* base, long long plane_stride, int c,
                                         long long row, uint4* out) {
  constexpr int kP = Elem<T>::kPerRecord;
  const unsigned char* q = base + static_cast<long long>(c / kP) * plane_stride + row * 16;
  out[0] = *reinterpret_cast<const uint4*>(q);
  if constexpr (kP == 4) out[1] = *reinterpret_cast<const uint4*>(q + plane_stride);
}

template <typename T>
__device__ __forceinline__ void unpackRec8(const uint4* in, float* v) {
  if constexpr (Elem<T>::kTf32) {
    const float4 a = *reinterpret_cast<const float4*>(&in[0]);
    const float4 b = *reinterpret_cast<const float4*>(&in[1]);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    unpack8<T>(in[0], v);
  }
}

template <typename T>
__device__ __forceinline__ void storeRec8(unsigned char* base, long long plane_stride, int c,
                                          long long row, const float* v, bool exact) {
  constexpr int kP = Elem<T>::kPerRecord;
  unsigned char* q = base + static_cast<long long>(c / kP) * plane_stride + row * 16;
  if constexpr (Elem<T>::kTf32) {
    if (exact) {  // FPK_DTYPE_F32_EXACT: the value as accumulated
      *reinterpret_cast<float4*>(q) = make_float4(v[0], v[1], v[2], v[3]);
      *reinterpret_cast<float4*>(q + plane_stride) = make_float4(v[4], v[5], v[6], v[7]);
      return;
    }
    // fp32 outputs are the next layer's TF32 operands: round to nearest here.
    *reinterpret_cast<float4*>(q) = make_float4(tf32Round(v[0]), tf32Round(v[1]), tf32Round(v[2]), tf32Round(v[3]));
    *reinterpret_cast<float4*>(q + plane_stride) =
        make_float4(tf32Round(v[4]), tf32Round(v[5]), tf32Round(v[6]), tf32Round(v[7]));
  } else {
    (void)exact;
    *reinterpret_cast<uint4*>(q) = pack8<T>(v);
  }
}

// Where output row r lands in the layer's destination layout (see include/fpk.h).
struct RowDst {
  bool valid;
  long long drow;
  int ch_base;
  int pos_row;
};

__device__ __forceinline__ RowDst rowDst(const fpk_gemm_desc_t& d, int r) {
  RowDst o{r < d.rows, 0, 0, 0};
  if (!o.valid) return o;
  const int img = r / d.img_rows;
  const int loc = r - img * d.img_rows;
  const int gy = loc / d.grid_w;
  const int gx = loc - gy * d.grid_w;
  o.valid = gy < d.valid_h && gx < d.valid_w;
  switch (d.dst_mode) {
    case FPK_DST_S2D:
      o.drow = static_cast<long long>(img) * d.dst_img_rows + ((gy + 1) >> 1) * d.dst_grid_w + ((gx + 1) >> 1);
      o.ch_base = (((gy + 1) & 1) * 2 + ((gx + 1) & 1)) * d.cout;
      break;
    case FPK_DST_CONCAT:
      o.drow = static_cast<long long>(img % d.img_mod) * d.img_rows + loc;
      o.ch_base = (img / d.img_mod) * d.ch_step;
      break;
    case FPK_DST_TOKENS:
      o.drow = static_cast<long long>(img) * d.valid_h * d.valid_w + gy * d.valid_w + gx;
      o.pos_row = gy * d.valid_w + gx;
      break;
    default:
      o.drow = r;
  }
  return o;
}

// Bias / residual / ReLU / positional embedding on the accumulator values of
// output channels n..n+7 of one row, stored into the destination layout.
template <typename T>
__device__ __forceinline__ void apply8(const fpk_gemm_desc_t& d, const RowDst& rd, float* v, int n,
                                       const uint4* res_rec, bool has_res) {
  if (d.bias != nullptr) {
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(d.bias + n));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(d.bias + n + 4));
    v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
    v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
  }
  if (has_res) {
    float rf[8];
    unpackRec8<T>(res_rec, rf);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] += rf[e];
  }
  if (d.relu) {
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = fmaxf(v[e], 0.0f);
  }
  if (d.dst_mode == FPK_DST_TOKENS && d.pos != nullptr) {
    const float* pp = d.pos + static_cast<long long>(rd.pos_row) * d.cout + n;
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] += __ldg(pp + e);
  }
}

template <typename T>
__device__ __forceinline__ void finish8(const fpk_gemm_desc_t& d, const RowDst& rd, float* v, int n,
                                        const uint4* res_rec, bool has_res) {
  apply8<T>(d, rd, v, n, res_rec, has_res);
  storeRec8<T>(static_cast<unsigned char*>(d.dst), d.dst_plane_stride, rd.ch_base + n, rd.drow, v,
               d.dtype == FPK_DTYPE_F32_EXACT);
}

// Split-K partial sums: split ks of output tile mn is a [BN/4][128][4] fp32
// block (column quads outermost, rows, then the 4 columns of a quad), so a
// warp's 32 consecutive rows read or write one contiguous 512-byte run.
__device__ __forceinline__ float4* splitPartial(const fpk_gemm_desc_t& d, const Plan& pl, int bn, int mn,
                                                int ks) {
  return static_cast<float4*>(d.splitk_ws) + (static_cast<size_t>(mn) * pl.k_splits + ks) * (bn / 4) * kBlockM;
}

// Second launch of a split-K layer: one thread per (row, 8 output channels)
// adds the k_splits partials in split order, then applies the layer's
// epilogue (bias, residual, ReLU, positional embedding, destination layout).
template <typename T>
__global__ void __launch_bounds__(256) splitReduceKernel(const fpk_gemm_desc_t d, const Plan pl, int bn) {
  pdlTrigger();
  pdlWait();  // every split of the GEMM launch has written its partials
  const int groups = bn / 8;
  const long long i = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;
  if (i >= static_cast<long long>(pl.m_tiles) * pl.n_tiles * groups * kBlockM) return;
  const int row = static_cast<int>(i % kBlockM);
  const long long t = i / kBlockM;
  const int cg = static_cast<int>(t % groups);
  const int mn = static_cast<int>(t / groups);
  const int r = (mn / pl.n_tiles) * kBlockM + row;
  const int n = (mn % pl.n_tiles) * bn + cg * 8;
  const RowDst rd = rowDst(d, r);
  if (!rd.valid) return;
  const float4* p = splitPartial(d, pl, bn, mn, 0) + static_cast<size_t>(cg * 2) * kBlockM + row;
  const size_t split_stride = static_cast<size_t>(bn / 4) * kBlockM;
  float4 lo[8], hi[8];
#pragma unroll
  for (int s = 0; s < 8; ++s) {
    if (s < pl.k_splits) {
      lo[s] = __ldcg(p + s * split_stride);
      hi[s] = __ldcg(p + s * split_stride + kBlockM);
    }
  }
  float v[8] = {lo[0].x, lo[0].y, lo[0].z, lo[0].w, hi[0].x, hi[0].y, hi[0].z, hi[0].w};
#pragma unroll
  for (int s = 1; s < 8; ++s) {
    if (s < pl.k_splits) {
      v[0] += lo[s].x; v[1] += lo[s].y; v[2] += lo[s].z; v[3] += lo[s].w;
      v[4] += hi[s].x; v[5] += hi[s].y; v[6] += hi[s].z; v[7] += hi[s].w;
    }
  }
  const bool has_res = d.residual != nullptr;
  uint4 rr[2] = {};
  if (has_res) loadRec8<T>(static_cast<const unsigned char*>(d.residual), d.res_plane_stride, n, r, rr);
  finish8<T>(d, rd, v, n, rr, has_res);
}

// Epilogue of one accumulator row: converts TMEM columns [j0, j0 + kSpan) of
// output row r (tile columns from n0) with bias / residual / ReLU / positional
// embedding and stores them into the destination layout of the layer. t_base
// is the TMEM address of this warp's lane quarter at column 0 of the row block.
template <typename T, int kSpan>
__device__ __forceinline__ void epilogueRow(const fpk_gemm_desc_t& d, uint32_t t_base, int r, int n0, int j0) {
  const unsigned char* res = static_cast<const unsigned char*>(d.residual);
  const RowDst rd = rowDst(d, r);
  const bool has_res = rd.valid && res != nullptr;
  // Residual rows of the next 32 columns are fetched while the current
  // 32 are converted and stored.
  uint4 rv[4][2] = {}, rn[4][2] = {};
  if (has_res) {
#pragma unroll
    for (int g = 0; g < 4; ++g) loadRec8<T>(res, d.res_plane_stride, n0 + j0 + g * 8, r, rv[g]);
  }
#pragma unroll 1
  for (int j = j0; j < j0 + kSpan; j += 32) {
    uint32_t acc[32];
    FPB_TMEM_LD32(t_base + j, acc);
    if (has_res && j + 32 < j0 + kSpan) {
#pragma unroll
      for (int g = 0; g < 4; ++g) loadRec8<T>(res, d.res_plane_stride, n0 + j + 32 + g * 8, r, rn[g]);
    }
    tmemWaitLd();
    if (rd.valid) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(acc[g * 8 + e]);
        finish8<T>(d, rd, v, n0 + j + g * 8, rv[g], has_res);
      }
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      rv[g][0] = rn[g][0];
      rv[g][1] = rn[g][1];
    }
  }
}

// Staged epilogue of a dense 16-bit layer (SAME layout, every row valid):
// like epilogueRow, but each 32-column chunk of the warp's 32 rows is packed
// into a 2 KB shared-memory tile ([4 planes][32 rows][16 B], two per warp,
// alternating) and written by one bulk tensor store issued by lane 0, instead
// of 16-byte stores from every thread (which set the pace of short-K layers).
// r0 = the warp's first output row (a multiple of 32); rows past the layer's
// end are clipped by the tensor map. `chunks` counts this warp's chunks so far.
template <typename T, int kSpan>
__device__ __forceinline__ void epilogueRowStaged(const fpk_gemm_desc_t& d, uint32_t t_base, int r, int n0, int j0,
                                                  unsigned char* stage, const CUtensorMap* tmap_out, int r0,
                                                  uint32_t& chunks) {
  static_assert(Elem<T>::kPerRecord == 8, "16-bit outputs only");
  const int lane = threadIdx.x & 31;
  const unsigned char* res = static_cast<const unsigned char*>(d.residual);
  const RowDst rd = rowDst(d, r);
  const bool has_res = rd.valid && res != nullptr;
  uint4 rv[4][2] = {}, rn[4][2] = {};
  if (has_res) {
#pragma unroll
    for (int g = 0; g < 4; ++g) loadRec8<T>(res, d.res_plane_stride, n0 + j0 + g * 8, r, rv[g]);
  }
#pragma unroll 1
  for (int j = j0; j < j0 + kSpan; j += 32) {
    uint32_t acc[32];
    FPB_TMEM_LD32(t_base + j, acc);
    if (has_res && j + 32 < j0 + kSpan) {
#pragma unroll
      for (int g = 0; g < 4; ++g) loadRec8<T>(res, d.res_plane_stride, n0 + j + 32 + g * 8, r, rn[g]);
    }
    unsigned char* sb = stage + (chunks & 1u) * 2048u;
    if (chunks >= 2) {
      // The store issued two chunks ago from this buffer has read it.
      if (lane == 0) bulkWaitRead<1>();
      __syncwarp();
    }
    tmemWaitLd();
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __uint_as_float(acc[g * 8 + e]);
      apply8<T>(d, rd, v, n0 + j + g * 8, rv[g], has_res);
      *reinterpret_cast<uint4*>(sb + g * 512 + lane * 16) = pack8<T>(v);
    }
    fenceProxyAsyncSmem();
    __syncwarp();
    if (lane == 0) {
      tmaStore2d(tmap_out, 2 * r0, (n0 + j) / 8, sb);
      bulkCommit();
    }
    ++chunks;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      rv[g][0] = rn[g][0];
      rv[g][1] = rn[g][1];
    }
  }
}

// MH = output row halves per tile: 1 -> 128 x BN tiles; 2 -> 256 x BN tiles
// whose two 128-row halves share every weight stage (two MMAs per K step into
// separate accumulators), halving weight traffic for the narrow layers.
template <typename T, int BN, int MH>
__global__ void __launch_bounds__(kThreads, 1)
    gemmKernel(const fpk_gemm_desc_t d, const Plan pl, const __grid_constant__ CUtensorMap tmap_w) {
  pdlTrigger();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // Dynamic shared memory: [B stages][A windows][barriers]; B stages need 1024 B alignment.
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* b_smem = base;
  unsigned char* a_smem = b_smem + static_cast<size_t>(pl.b_stages) * pl.b_stage_bytes;
  Smem* sm = reinterpret_cast<Smem*>(a_smem + static_cast<size_t>(pl.a_slots) * pl.a_win_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = d.error_flag;
  // Accumulator buffers: two (the epilogue of tile i overlaps the MMAs of
  // tile i+1) when they fit the 512 TMEM columns, else one (256-row tiles of
  // 256 columns, used for the 1x1 linears).
  constexpr int kBufs = 2 * MH * BN <= 512 ? 2 : 1;
  constexpr uint32_t kTmemCols = kBufs * MH * BN;
  constexpr int kTileM = kBlockM * MH;
  static_assert(kTmemCols <= 512, "accumulators exceed TMEM");

  if (threadIdx.x < pl.stages_per_chunk * 2) {
    // Descriptor start offsets of the two 32-byte K steps handled by this thread.
    constexpr int kStep = 32 / Elem<T>::kBytes;  // K elements per MMA
    const uint32_t plane_units = static_cast<uint32_t>(pl.win_rows);  // plane bytes / 16
    uint32_t packed = 0;
    for (int h = 0; h < 2; ++h) {
      const int k_local = (threadIdx.x * 2 + h) * kStep;
      const int tap = k_local / pl.cw;
      const int c = k_local - tap * pl.cw;
      const uint32_t off = static_cast<uint32_t>(d.tap_off[tap] - pl.min_off) +
                           static_cast<uint32_t>(c / Elem<T>::kPerRecord) * plane_units;
      packed |= (off & 0xFFFFu) << (16 * h);
    }
    reinterpret_cast<uint32_t*>(sm->a_off)[threadIdx.x] = packed;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbarInit(&sm->acc_full[i], 1);
      mbarInit(&sm->acc_empty[i], kEpilogueWarps);
    }
    for (int i = 0; i < pl.a_slots; ++i) {
      mbarInit(&sm->a_full[i], 1);
      mbarInit(&sm->a_empty[i], 1);
    }
    for (int i = 0; i < pl.b_stages; ++i) {
      mbarInit(&sm->b_full[i], 1);
      mbarInit(&sm->b_empty[i], 1);
    }
    mbarInit(&sm->drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smemU32(&sm->tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  tcFenceAfter();
  pdlWait();  // the previous layer's output (this layer's input) is complete from here on
  const uint32_t tmem = sm->tmem_base;
  // Work items: output tiles, each split into k_splits contiguous chunk ranges.
  const int n_tiles_total = pl.m_tiles * pl.n_tiles * pl.k_splits;
  const int taps_cw = d.taps * pl.cw;
  auto chunkRange = [&](int tile, int* c0, int* c1) {
    const int ks = tile % pl.k_splits;
    *c0 = ks * pl.n_chunks / pl.k_splits;
    *c1 = (ks + 1) * pl.n_chunks / pl.k_splits;
  };

  if (warp == 0) {
    {
      // ---------------- producer ----------------
      // The whole warp runs the loop; lane p issues the bulk copy of channel
      // plane p of each window, lane 0 arms the barriers and loads weights.
      const unsigned char* a_bytes = static_cast<const unsigned char*>(d.a);
      const uint32_t plane_bytes = static_cast<uint32_t>(pl.win_rows) * 16u;
      uint32_t a_iter = 0, b_iter = 0;
      int slot = 0, bs = 0;
      uint32_t a_phase = 0, b_phase = 0;
      // A withheld load (failure-injection test) leaves the MMA warp's first
      // `full` wait to run out: it records error 14 and every role exits.
      bool ok = pl.withhold_loads == 0;
      for (int tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x) {
        const int mn = tile / pl.k_splits;
        const int m0 = (mn / pl.n_tiles) * kTileM;
        const int n0 = (mn % pl.n_tiles) * BN;
        int c0, c1;
        chunkRange(tile, &c0, &c1);
        for (int ch = c0; ch < c1 && ok; ++ch) {
          ok = warpWaitBar(&sm->a_empty[slot], a_phase ^ 1, err, 11);
          if (!ok) break;
          if (lane == 0) mbarExpectTx(&sm->a_full[slot], pl.a_win_bytes);
          __syncwarp();
          unsigned char* win = a_smem + static_cast<size_t>(slot) * pl.a_win_bytes;
          const unsigned char* src = a_bytes + static_cast<long long>(ch * pl.planes) * d.a_plane_stride +
                                     static_cast<long long>(m0 + pl.min_off) * 16;
          for (int p = lane; p < pl.planes; p += 32) {
            bulkCopy(win + p * plane_bytes, src + static_cast<long long>(p) * d.a_plane_stride, plane_bytes,
                     &sm->a_full[slot]);
          }
          ++a_iter;
          if (++slot == pl.a_slots) { slot = 0; a_phase ^= 1; }
          for (int st = 0; st < pl.stages_per_chunk; ++st) {
            ok = warpWaitBar(&sm->b_empty[bs], b_phase ^ 1, err, 12);
            if (!ok) break;
            if (lane == 0) {
              mbarExpectTx(&sm->b_full[bs], pl.b_stage_bytes);
              tmaLoad2d(b_smem + static_cast<size_t>(bs) * pl.b_stage_bytes, &tmap_w,
                        ch * taps_cw + st * Elem<T>::kPerStage, n0, &sm->b_full[bs]);
            }
            ++b_iter;
            if (++bs == pl.b_stages) { bs = 0; b_phase ^= 1; }
          }
        }
      }
      // Drain: every load armed above must land before the CTA may exit.
      if (lane == 0) {
        const uint32_t na = static_cast<uint32_t>(pl.a_slots);
        for (uint32_t i = a_iter > na ? a_iter - na : 0; i < a_iter; ++i) {
          drainBar(&sm->a_full[i % na], (i / na) & 1);
        }
        const uint32_t nb = static_cast<uint32_t>(pl.b_stages);
        for (uint32_t i = b_iter > nb ? b_iter - nb : 0; i < b_iter; ++i) {
          drainBar(&sm->b_full[i % nb], (i / nb) & 1);
        }
      }
    }
  } else if (warp == 1) {
    {
      // ---------------- MMA issuer ----------------
      // Descriptors are built once; per K=16 step only the 14-bit start
      // address field changes (an add that cannot carry: every start is a
      // valid shared-memory address below 2^18 bytes).
      const uint32_t idesc = Elem<T>::instrDesc(BN, kBlockM);
      const uint64_t a_desc0 =
          smemDesc(smemU32(a_smem), static_cast<uint32_t>(pl.win_rows) * 16u, 128u, kLayoutNone);
      const uint64_t b_desc0 = smemDesc(smemU32(b_smem), 16u, 1024u, kLayoutSw128);
      const uint32_t a_slot_units = pl.a_win_bytes >> 4;
      const uint32_t b_stage_units = pl.b_stage_bytes >> 4;
      int slot = 0, bs = 0;
      uint32_t a_phase = 0, b_phase = 0, t_iter = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < n_tiles_total && ok; tile += gridDim.x, ++t_iter) {
        const int buf = static_cast<int>(t_iter % kBufs);
        ok = warpWaitBar(&sm->acc_empty[buf], ((t_iter / kBufs) & 1) ^ 1, err, 13);
        if (!ok) break;
        tcFenceAfter();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(buf * MH * BN);
        uint32_t accumulate = 0;
        int c0, c1;
        chunkRange(tile, &c0, &c1);
        for (int ch = c0; ch < c1 && ok; ++ch) {
          ok = warpWaitBar(&sm->a_full[slot], a_phase, err, 14);
          if (!ok) break;
          tcFenceAfter();
          const uint64_t a_base = a_desc0 + static_cast<uint64_t>(slot) * a_slot_units;
          for (int st = 0; st < pl.stages_per_chunk; ++st) {
            const uint2 offs = sm->a_off[st];  // read before the wait: it does not depend on the stage
            ok = warpWaitBar(&sm->b_full[bs], b_phase, err, 15);
            if (!ok) break;
            tcFenceAfter();
            const uint64_t b_base = b_desc0 + static_cast<uint64_t>(bs) * b_stage_units;
#pragma unroll
            for (int h = 0; h < MH; ++h) {
              // Half h reads the window 128 rows (128 x 16 B = 128 units) further on.
              const uint64_t ah = a_base + static_cast<uint64_t>(h * 128);
              const uint32_t dh = d_tmem + static_cast<uint32_t>(h * BN);
              mmaTElect<T>(dh, ah + (offs.x & 0xFFFFu), b_base, idesc, accumulate);
              mmaTElect<T>(dh, ah + (offs.x >> 16), b_base + 2, idesc, 1u);
              mmaTElect<T>(dh, ah + (offs.y & 0xFFFFu), b_base + 4, idesc, 1u);
              mmaTElect<T>(dh, ah + (offs.y >> 16), b_base + 6, idesc, 1u);
            }
            accumulate = 1u;
            tcCommitElect(&sm->b_empty[bs]);
            if (++bs == pl.b_stages) { bs = 0; b_phase ^= 1; }
          }
          tcCommitElect(&sm->a_empty[slot]);
          if (++slot == pl.a_slots) { slot = 0; a_phase ^= 1; }
        }
        // A tile whose operand wait gave up is never handed to the epilogue:
        // its warps see the error flag and exit without storing.
        if (ok) tcCommitElect(&sm->acc_full[buf]);
      }
      // Drain: wait until every MMA issued above has completed (also after an
      // error: TMEM is released only once no MMA can still write it).
      tcCommitElect(&sm->drain);
      drainBar(&sm->drain, 0);
    }
  } else {
    // ---------------- epilogue (warps 2..9) ----------------
    const int quarter = warp & 3;    // TMEM lane quarter this warp may access
    const int pair = (warp - 2) >> 2;  // MH=1: half of the BN columns; MH=2: row half
    constexpr int kSpan = MH == 1 ? BN / 2 : BN;  // columns converted by one warp
    const int m_half = MH == 1 ? 0 : pair;
    const int row_in_tile = m_half * kBlockM + quarter * 32 + lane;
    uint32_t t_iter = 0;
    for (int tile = blockIdx.x; tile < n_tiles_total; tile += gridDim.x, ++t_iter) {
      const int mn = tile / pl.k_splits;
      const int m0 = (mn / pl.n_tiles) * kTileM;
      const int n0 = (mn % pl.n_tiles) * BN;
      const int buf = static_cast<int>(t_iter % kBufs);
      if (!waitBar(&sm->acc_full[buf], (t_iter / kBufs) & 1, err, 17)) break;
      tcFenceAfter();
      const uint32_t t_base =
          tmem + (static_cast<uint32_t>(quarter * 32) << 16) +
          static_cast<uint32_t>((buf * MH + m_half) * BN);
      const int j0 = MH == 1 ? pair * kSpan : 0;
      if (MH == 1 && pl.k_splits > 1) {
        // Split K: this warp's 32 rows x kSpan columns of the partial sum go
        // to the scratch; the reduce launch adds the splits and stores.
        float4* own = splitPartial(d, pl, BN, mn, tile % pl.k_splits) + row_in_tile;
#pragma unroll 1
        for (int j = j0; j < j0 + kSpan; j += 32) {
          uint32_t acc[32];
          FPB_TMEM_LD32(t_base + j, acc);
          tmemWaitLd();
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            __stcg(own + static_cast<size_t>((j >> 2) + q) * kBlockM,
                   make_float4(__uint_as_float(acc[4 * q]), __uint_as_float(acc[4 * q + 1]),
                               __uint_as_float(acc[4 * q + 2]), __uint_as_float(acc[4 * q + 3])));
          }
        }
        tcFenceBefore();
        __syncwarp();
        if (lane == 0) mbarArrive(&sm->acc_empty[buf]);
        continue;
      }
      epilogueRow<T, kSpan>(d, t_base, m0 + row_in_tile, n0, j0);
      tcFenceBefore();
      __syncwarp();
      if (lane == 0) mbarArrive(&sm->acc_empty[buf]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    tcFenceAfter();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(kTmemCols));
  }
}

// CTA-pair variant (clusters of two CTAs, tcgen05 cta_group::2). A pair owns
// tiles of 2 * MH * 128 rows x BN channels: CTA r (r = 0 leader, 1 peer)
// stages the activation window of its MH * 128 rows and weight rows
// n0 + r BN/2 .. + BN/2 in its own shared memory, and the leader's MMA lane
// issues, per K step and row half h < MH, an M=256 x N=BN MMA that reads
// 128 rows of A from each CTA and B half from each; accumulator rows of CTA r
// land in its own TMEM (MH blocks of BN columns per buffer). Per SM this
// halves the weight bytes staged and read per MMA, which is what limits the
// single-CTA tiles (shared-memory bandwidth), and leaves room for two
// accumulator buffers. BN = 256 with MH = 1, or BN = 128 with MH = 2.
//   * both producers wait on their own `empty` barriers (the leader's commits
//     signal both CTAs) and count their tile loads on the leader's `full`
//     barriers, which the leader arms with the bytes of both CTAs;
//   * both CTAs' epilogues wait on their own `acc_full` (signalled by the
//     leader's commit) and release the buffer on the leader's `acc_empty`.
// Activation windows are row-run TMA tiles (a plane's rows as one contiguous
// run of 8-byte elements, zero fill outside the tensor): one box of all
// planes for windows of at most 128 rows, else per plane boxes of 128 rows
// and a tail box, issued by parallel lanes.
template <typename T, int BN, int MH>
__global__ void __launch_bounds__(kThreads, 1)
    gemmPairKernel(const fpk_gemm_desc_t d, const Plan pl, const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_a_tail,
                   const __grid_constant__ CUtensorMap tmap_out) {
  pdlTrigger();
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  unsigned char* b_smem = base;
  unsigned char* a_smem = b_smem + static_cast<size_t>(pl.b_stages) * pl.b_stage_bytes;
  Smem* sm = reinterpret_cast<Smem*>(a_smem + static_cast<size_t>(pl.a_slots) * pl.a_slot_bytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = clusterCtaRank();
  const bool leader = rank == 0;
  int* err = d.error_flag;
  constexpr uint32_t kTmemCols = 2 * MH * BN;  // two accumulator buffers of MH blocks of 128 lanes x BN
  constexpr int kCtaM = MH * kBlockM;          // output rows per CTA per tile
  constexpr int kPairM = 2 * kCtaM;
  static_assert(kTmemCols <= 512, "accumulators exceed TMEM");

  if (threadIdx.x < pl.stages_per_chunk * 2) {
    constexpr int kStep = 32 / Elem<T>::kBytes;
    const uint32_t plane_units = pl.a_plane_pitch >> 4;
    uint32_t packed = 0;
    for (int h = 0; h < 2; ++h) {
      const int k_local = (threadIdx.x * 2 + h) * kStep;
      const int tap = k_local / pl.cw;
      const int c = k_local - tap * pl.cw;
      const uint32_t off = static_cast<uint32_t>(d.tap_off[tap] - pl.min_off) +
                           static_cast<uint32_t>(c / Elem<T>::kPerRecord) * plane_units;
      packed |= (off & 0xFFFFu) << (16 * h);
    }
    reinterpret_cast<uint32_t*>(sm->a_off)[threadIdx.x] = packed;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbarInit(&sm->acc_full[i], 1);
      mbarInit(&sm->acc_empty[i], 2 * kEpilogueWarps);
    }
    for (int i = 0; i < pl.a_slots; ++i) {
      mbarInit(&sm->a_full[i], 1);
      mbarInit(&sm->a_empty[i], 1);
    }
    for (int i = 0; i < pl.b_stages; ++i) {
      mbarInit(&sm->b_full[i], 1);
      mbarInit(&sm->b_empty[i], 1);
    }
    mbarInit(&sm->drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smemU32(&sm->tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  __syncthreads();
  tcFenceBefore();
  // Both CTAs' barriers are initialised and both TMEM allocations made before
  // any thread signals the peer or any MMA writes the peer's TMEM.
  clusterSync();
  tcFenceAfter();
  pdlWait();  // the previous layer's output (this layer's input) is complete from here on
  const uint32_t tmem = sm->tmem_base;
  const int n_tiles_total = pl.m_tiles * pl.n_tiles;
  const int pair_id = static_cast<int>(blockIdx.x >> 1);
  const int n_pairs = static_cast<int>(gridDim.x >> 1);
  const int taps_cw = d.taps * pl.cw;

  if (warp == 0) {
    {
      // ---------------- producer (both CTAs; whole warp, lane 0 issues) ----------------
      int slot = 0, bs = 0;
      uint32_t a_phase = 0, b_phase = 0, a_iter = 0, b_iter = 0;
      bool ok = true;
      const int row_off = static_cast<int>(rank) * kCtaM + pl.min_off;
      const int n_off = static_cast<int>(rank) * (BN / 2);
      for (int tile = pair_id; tile < n_tiles_total && ok; tile += n_pairs) {
        const int m0 = (tile / pl.n_tiles) * kPairM;
        const int n0 = (tile % pl.n_tiles) * BN;
        for (int ch = 0; ch < pl.n_chunks && ok; ++ch) {
          ok = warpWaitBar(&sm->a_empty[slot], a_phase ^ 1, err, 21);
          if (!ok) break;
          // The window as row-run tiles (each plane's rows are one contiguous
          // run): one box of every plane when it has at most 128 rows, else
          // per plane ceil(rows / 128) boxes (the last one the tail map's
          // size), lane c * planes + p issuing box c of plane p.
          if (lane == 0 && leader) mbarExpectTx(&sm->a_full[slot], 2u * pl.a_win_bytes);
          __syncwarp();
          {
            unsigned char* win = a_smem + static_cast<size_t>(slot) * pl.a_slot_bytes;
            const uint32_t bar = mapaShared(smemU32(&sm->a_full[slot]), 0);
            const int row = m0 + row_off;
            if (pl.win_rows <= 128) {
              if (lane == 0) tmaLoad2dPair(win, &tmap_a, 2 * row, ch * pl.planes, bar);
            } else {
              const int n_box = (pl.win_rows + 127) / 128;
              if (lane < n_box * pl.planes) {
                const int c = lane / pl.planes;
                const int p = lane - c * pl.planes;
                const bool tail = c == n_box - 1 && (pl.win_rows & 127) != 0;
                tmaLoad2dPair(win + static_cast<size_t>(p) * pl.a_plane_pitch + static_cast<size_t>(c) * 128 * 16,
                              tail ? &tmap_a_tail : &tmap_a, 2 * (row + 128 * c), ch * pl.planes + p, bar);
              }
            }
          }
          ++a_iter;
          if (++slot == pl.a_slots) { slot = 0; a_phase ^= 1; }
          for (int st = 0; st < pl.stages_per_chunk; ++st) {
            ok = warpWaitBar(&sm->b_empty[bs], b_phase ^ 1, err, 22);
            if (!ok) break;
            if (lane == 0) {
              if (leader) mbarExpectTx(&sm->b_full[bs], 2u * pl.b_stage_bytes);
              tmaLoad2dPair(b_smem + static_cast<size_t>(bs) * pl.b_stage_bytes, &tmap_w,
                            ch * taps_cw + st * Elem<T>::kPerStage, n0 + n_off,
                            mapaShared(smemU32(&sm->b_full[bs]), 0));
            }
            ++b_iter;
            if (++bs == pl.b_stages) { bs = 0; b_phase ^= 1; }
          }
        }
      }
      // Drain: the last use of every slot and stage must have been consumed by
      // the leader's MMAs (which implies its loads landed) before the CTA exits.
      if (lane == 0) {
        const uint32_t na = static_cast<uint32_t>(pl.a_slots);
        for (uint32_t i = a_iter > na ? a_iter - na : 0; i < a_iter; ++i) {
          drainBar(&sm->a_empty[i % na], (i / na) & 1);
        }
        const uint32_t nb = static_cast<uint32_t>(pl.b_stages);
        for (uint32_t i = b_iter > nb ? b_iter - nb : 0; i < b_iter; ++i) {
          drainBar(&sm->b_empty[i % nb], (i / nb) & 1);
        }
      }
    }
  } else if (warp == 1) {
    if (leader) {
      // ---------------- MMA issuer (leader CTA) ----------------
      const uint32_t idesc = Elem<T>::instrDesc(BN, 2 * kBlockM);  // every pair MMA is M = 256
      const uint64_t a_desc0 =
          smemDesc(smemU32(a_smem), pl.a_plane_pitch, 128u, kLayoutNone);
      const uint64_t b_desc0 = smemDesc(smemU32(b_smem), 16u, 1024u, kLayoutSw128);
      const uint32_t a_slot_units = pl.a_slot_bytes >> 4;
      const uint32_t b_stage_units = pl.b_stage_bytes >> 4;
      int slot = 0, bs = 0;
      uint32_t a_phase = 0, b_phase = 0, t_iter = 0;
      bool ok = true;
      for (int tile = pair_id; tile < n_tiles_total && ok; tile += n_pairs, ++t_iter) {
        const int buf = static_cast<int>(t_iter & 1);
        ok = warpWaitBar(&sm->acc_empty[buf], ((t_iter >> 1) & 1) ^ 1, err, 23);
        if (!ok) break;
        tcFenceAfter();
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(buf * MH * BN);
        uint32_t accumulate = 0;
        for (int ch = 0; ch < pl.n_chunks && ok; ++ch) {
          ok = warpWaitBar(&sm->a_full[slot], a_phase, err, 24);
          if (!ok) break;
          tcFenceAfter();
          const uint64_t a_base = a_desc0 + static_cast<uint64_t>(slot) * a_slot_units;
          for (int st = 0; st < pl.stages_per_chunk; ++st) {
            const uint2 offs = sm->a_off[st];  // read before the wait: it does not depend on the stage
            ok = warpWaitBar(&sm->b_full[bs], b_phase, err, 25);
            if (!ok) break;
            tcFenceAfter();
            const uint64_t b_base = b_desc0 + static_cast<uint64_t>(bs) * b_stage_units;
#pragma unroll
            for (int h = 0; h < MH; ++h) {
              // Row half h reads the window 128 rows (128 units of 16 B) further on.
              const uint64_t ah = a_base + static_cast<uint64_t>(h * 128);
              const uint32_t dh = d_tmem + static_cast<uint32_t>(h * BN);
              if constexpr (Elem<T>::kTf32) {
                tcMmaPairTf32Elect(dh, ah + (offs.x & 0xFFFFu), b_base, idesc, accumulate);
                tcMmaPairTf32Elect(dh, ah + (offs.x >> 16), b_base + 2, idesc, 1u);
                tcMmaPairTf32Elect(dh, ah + (offs.y & 0xFFFFu), b_base + 4, idesc, 1u);
                tcMmaPairTf32Elect(dh, ah + (offs.y >> 16), b_base + 6, idesc, 1u);
              } else {
                tcMmaPairF16Elect(dh, ah + (offs.x & 0xFFFFu), b_base, idesc, accumulate);
                tcMmaPairF16Elect(dh, ah + (offs.x >> 16), b_base + 2, idesc, 1u);
                tcMmaPairF16Elect(dh, ah + (offs.y & 0xFFFFu), b_base + 4, idesc, 1u);
                tcMmaPairF16Elect(dh, ah + (offs.y >> 16), b_base + 6, idesc, 1u);
              }
            }
            accumulate = 1u;
            tcCommitPairBothElect(&sm->b_empty[bs]);
            if (++bs == pl.b_stages) { bs = 0; b_phase ^= 1; }
          }
          tcCommitPairBothElect(&sm->a_empty[slot]);
          if (++slot == pl.a_slots) { slot = 0; a_phase ^= 1; }
        }
        if (ok) tcCommitPairBothElect(&sm->acc_full[buf]);  // as in gemmKernel: no partial tile is stored
      }
      tcCommitPairOwnElect(&sm->drain);
      drainBar(&sm->drain, 0);  // as in gemmKernel: no MMA in flight past this point
    }
  } else {
    // ---------------- epilogue (warps 2..9, both CTAs) ----------------
    const int quarter = warp & 3;
    const int pair = (warp - 2) >> 2;  // MH=1: half of the BN columns; MH=2: row half
    constexpr int kSpan = MH == 1 ? BN / 2 : BN;  // columns converted by one warp
    const int m_half = MH == 1 ? 0 : pair;
    const int row_in_tile = static_cast<int>(rank) * kCtaM + m_half * kBlockM + quarter * 32 + lane;
    unsigned char* stage = base + pl.stage_off + static_cast<size_t>(warp - 2) * 4096;
    uint32_t chunks = 0;
    uint32_t t_iter = 0;
    for (int tile = pair_id; tile < n_tiles_total; tile += n_pairs, ++t_iter) {
      const int m0 = (tile / pl.n_tiles) * kPairM;
      const int n0 = (tile % pl.n_tiles) * BN;
      const int buf = static_cast<int>(t_iter & 1);
      if (!waitBar(&sm->acc_full[buf], (t_iter >> 1) & 1, err, 27)) break;
      tcFenceAfter();
      const uint32_t t_base =
          tmem + (static_cast<uint32_t>(quarter * 32) << 16) + static_cast<uint32_t>((buf * MH + m_half) * BN);
      bool staged = false;
      if constexpr (!Elem<T>::kTf32) {
        if (pl.tma_store) {
          epilogueRowStaged<T, kSpan>(d, t_base, m0 + row_in_tile, n0, MH == 1 ? pair * kSpan : 0, stage, &tmap_out,
                                      m0 + row_in_tile - lane, chunks);
          staged = true;
        }
      }
      if (!staged) epilogueRow<T, kSpan>(d, t_base, m0 + row_in_tile, n0, MH == 1 ? pair * kSpan : 0);
      tcFenceBefore();
      __syncwarp();
      if (lane == 0) mbarArriveCluster(mapaShared(smemU32(&sm->acc_empty[buf]), 0));
    }
    // Every bulk store this warp issued has completed before the CTA exits.
    if (lane == 0 && chunks > 0) bulkWaitAll();
    __syncwarp();
  }
  __syncthreads();
  tcFenceBefore();
  // Neither CTA frees its TMEM (or exits) while the leader's MMAs or the
  // peer's signals may still touch it.
  clusterSync();
  if (warp == 1) {
    tcFenceAfter();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Host side: tensor maps, planning, launch.
// ---------------------------------------------------------------------------

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encodeFn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<EncodeTiledFn>(p);
    }
  });
  return fn;
}

int makeWeightMap(const fpk_gemm_desc_t& d, int kprime, int bn, CUtensorMap* map) {
  EncodeTiledFn enc = encodeFn();
  if (enc == nullptr) return fail("fpk_gemm: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(kprime), static_cast<cuuint64_t>(d.cout)};
  const bool f32 = d.dtype == FPK_DTYPE_F32 || d.dtype == FPK_DTYPE_F32_EXACT;
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(kprime) * (f32 ? 4 : 2)};
  const int esize = f32 ? 4 : 2;
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kStageBytes / esize), static_cast<cuuint32_t>(bn)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map,
                         d.dtype == FPK_DTYPE_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                         : f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                         2, const_cast<void*>(d.w), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail("fpk_gemm: cuTensorMapEncodeTiled failed (" + std::to_string(r) + ")");
  return 0;
}

// Splits the shared memory left after the barriers between activation window
// slots and weight stages so that the MMAs can run furthest ahead of the
// loads: the number of weight stages covered by both the window slots in
// flight (slots x stages per window) and the weight stages themselves.
// Convolutions (many stages per window) end up with two slots; 1x1 layers (one
// stage per window) with as many slots as stages. Returns false if fewer than
// two of each fit.
bool chooseSlots(uint32_t slot_bytes, uint32_t stage_bytes, int stages_per_chunk, int* slots_out,
                 int* stages_out, size_t reserve = 0) {
  int best = -1;
  for (int slots = 2; slots <= kMaxASlots; ++slots) {
    const size_t used = 1024 + sizeof(Smem) + reserve + static_cast<size_t>(slots) * slot_bytes;
    if (used >= kSmemBytes) break;
    int stages = static_cast<int>((kSmemBytes - used) / stage_bytes);
    stages = stages > kMaxBStages ? kMaxBStages : stages;
    if (stages < 2) break;
    const int depth = slots * stages_per_chunk < stages ? slots * stages_per_chunk : stages;
    if (depth > best) {
      best = depth;
      *slots_out = slots;
      *stages_out = stages;
    }
  }
  return best > 0;
}

// SM count of the current device (cached per device).
int numSms() {
  static DeviceValue cache;
  return cache.get([](int dev) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  });
}

template <typename T, int BN, int MH>
int launch(const fpk_gemm_desc_t& d, const Plan& pl, const CUtensorMap& map, size_t smem,
           cudaStream_t stream) {
  static DeviceOnce smem_attr;
  const cudaError_t ae = smem_attr.run([] {
    return cudaFuncSetAttribute(gemmKernel<T, BN, MH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kSmemBytes));
  });
  if (ae != cudaSuccess) {
    cudaGetLastError();
    return fail(std::string("fpk_gemm smem attribute: ") + cudaGetErrorString(ae));
  }
  const int tiles = pl.m_tiles * pl.n_tiles * pl.k_splits;
  const int grid = tiles < numSms() ? tiles : numSms();
  prof::countLaunch(prof::kGemm);
  cudaError_t e = launchPdl(gemmKernel<T, BN, MH>, dim3(grid), dim3(kThreads), smem, stream, d, pl, map);
  if (e == cudaSuccess && pl.k_splits > 1) {
    prof::countLaunch(prof::kGemm);
    const long long threads = static_cast<long long>(pl.m_tiles) * pl.n_tiles * (BN / 8) * kBlockM;
    e = launchPdl(splitReduceKernel<T>, dim3(static_cast<unsigned>((threads + 255) / 256)), dim3(256), 0, stream, d,
                  pl, BN);
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(std::string("gemmKernel launch: ") + cudaGetErrorString(e));
  }
  return checkLaunch("gemmKernel");
}

std::atomic<bool> g_cta_pairs{true};
std::atomic<bool> g_withhold_loads{false};
std::atomic<bool> g_tma_store{true};
template <typename T, int BN, int MH>
int launchPair(const fpk_gemm_desc_t& d, const Plan& pl, const CUtensorMap& map_w, const CUtensorMap& map_a,
               const CUtensorMap& map_a_tail, const CUtensorMap& map_out, size_t smem, cudaStream_t stream) {
  static DeviceOnce smem_attr;
  static std::mutex mu;
  static std::unordered_map<long long, int> clusters_for;  // (device, smem) -> co-resident pairs
  const int dev = currentDevice();
  const cudaError_t ae = smem_attr.run([] {
    return cudaFuncSetAttribute(gemmPairKernel<T, BN, MH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(kSmemBytes));
  });
  if (ae != cudaSuccess) {
    cudaGetLastError();
    return fail(std::string("fpk_gemm (pairs) smem attribute: ") + cudaGetErrorString(ae));
  }
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see fp_launch.hpp
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;  // the occupancy query below takes the cluster shape only
  int clusters = 0;
  {
    std::lock_guard<std::mutex> lock(mu);
    const long long key = (static_cast<long long>(dev) << 32) | static_cast<long long>(smem);
    auto it = clusters_for.find(key);
    if (it == clusters_for.end()) {
      cfg.gridDim = dim3(2 * (numSms() / 2));
      if (cudaOccupancyMaxActiveClusters(&clusters, gemmPairKernel<T, BN, MH>, &cfg) != cudaSuccess || clusters < 1) {
        cudaGetLastError();
        clusters = numSms() / 2;
      }
      clusters_for.emplace(key, clusters);
    } else {
      clusters = it->second;
    }
  }
  const int tiles = pl.m_tiles * pl.n_tiles;
  cfg.gridDim = dim3(2 * (tiles < clusters ? tiles : clusters));
  cfg.numAttrs = 2;
  prof::countLaunch(prof::kGemm);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, gemmPairKernel<T, BN, MH>, d, pl, map_w, map_a, map_a_tail, map_out);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(std::string("gemmPairKernel launch: ") + cudaGetErrorString(e));
  }
  return checkLaunch("gemmPairKernel");
}

template <typename T>
int launchShape(const fpk_gemm_desc_t& d, const Plan& pl, const CUtensorMap& map, size_t smem,
                cudaStream_t s, int bn, int mh) {
  if (mh == 2) {
    switch (bn) {
      case 64:
        return launch<T, 64, 2>(d, pl, map, smem, s);
      case 128:
        return launch<T, 128, 2>(d, pl, map, smem, s);
      default:
        return launch<T, 256, 2>(d, pl, map, smem, s);
    }
  }
  switch (bn) {
    case 64:
      return launch<T, 64, 1>(d, pl, map, smem, s);
    case 128:
      return launch<T, 128, 1>(d, pl, map, smem, s);
    default:
      return launch<T, 256, 1>(d, pl, map, smem, s);
  }
}

}  // namespace gemm

int makePlanarRowsMap(const void* base, long long rows, int planes, long long plane_stride, int box_rows,
                      int box_planes, CUtensorMap* map, const char* who) {
  gemm::EncodeTiledFn enc = gemm::encodeFn();
  if (enc == nullptr) return fail(std::string(who) + ": cuTensorMapEncodeTiled unavailable");
  if (box_rows <= 0 || box_rows > 128) return fail(std::string(who) + ": planar row box must be 1..128 rows");
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(2 * rows), static_cast<cuuint64_t>(planes)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(plane_stride)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(2 * box_rows), static_cast<cuuint32_t>(box_planes)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(std::string(who) + ": cuTensorMapEncodeTiled (planar rows) failed (" + std::to_string(r) + ")");
  }
  return 0;
}

}  // namespace fpb

using namespace fpb;

extern "C" int fpk_gemm(const fpk_gemm_desc_t* desc, void* stream) {
  using namespace fpb::gemm;
  if (desc == nullptr || desc->a == nullptr || desc->w == nullptr || desc->dst == nullptr ||
      desc->error_flag == nullptr) {
    return fail("fpk_gemm: null pointer in descriptor");
  }
  const fpk_gemm_desc_t& d = *desc;
  if (d.dtype != FPK_DTYPE_F16 && d.dtype != FPK_DTYPE_BF16 && d.dtype != FPK_DTYPE_F32 &&
      d.dtype != FPK_DTYPE_F32_EXACT) {
    return fail("fpk_gemm: dtype must be f16, bf16, f32 or f32-exact (TF32 tensor-core math)");
  }
  const int esize = (d.dtype == FPK_DTYPE_F32 || d.dtype == FPK_DTYPE_F32_EXACT) ? 4 : 2;
  const int stage_elems = kStageBytes / esize;  // 64 (16-bit) or 32 (fp32) channels per chunk
  if (d.taps < 1 || d.taps > FPK_GEMM_MAX_TAPS) return fail("fpk_gemm: taps out of range");
  if (d.cin < 32 || (d.cin != 32 && d.cin % stage_elems != 0)) {
    return fail("fpk_gemm: cin must be 32 or a multiple of 64 (16-bit) / 32 (f32)");
  }
  if (d.rows <= 0 || d.img_rows <= 0 || d.grid_w <= 0) return fail("fpk_gemm: bad grid");
  if (reinterpret_cast<uintptr_t>(d.a) % 16 || d.a_plane_stride % 16 ||
      reinterpret_cast<uintptr_t>(d.dst) % 16 || d.dst_plane_stride % 16 ||
      reinterpret_cast<uintptr_t>(d.w) % 16 || (d.bias && reinterpret_cast<uintptr_t>(d.bias) % 16)) {
    return fail("fpk_gemm: pointers and plane strides must be 16-byte aligned");
  }
  Plan pl{};
  pl.k_splits = 1;
  pl.cw = d.cin < stage_elems ? d.cin : stage_elems;
  pl.planes = pl.cw * esize / 16;
  pl.n_chunks = d.cin / pl.cw;
  if ((d.taps * pl.cw) % stage_elems != 0) return fail("fpk_gemm: taps*chunk must fill whole 128-byte stages");
  pl.stages_per_chunk = d.taps * pl.cw / stage_elems;
  if (pl.stages_per_chunk > kMaxStagesPerChunk) return fail("fpk_gemm: too many weight stages per chunk");
  int mn = d.tap_off[0], mx = d.tap_off[0];
  for (int t = 1; t < d.taps; ++t) {
    mn = d.tap_off[t] < mn ? d.tap_off[t] : mn;
    mx = d.tap_off[t] > mx ? d.tap_off[t] : mx;
  }
  int bn = d.cout >= 256 ? 256 : d.cout;
  if (d.cout % bn != 0 || (bn != 64 && bn != 128 && bn != 256)) {
    return fail("fpk_gemm: cout must be 64, 128 or a multiple of 256");
  }
  pl.min_off = mn;
  pl.b_stage_bytes = static_cast<uint32_t>(bn) * 128u;
  // Shared-memory plan for tiles of 128 * mh rows: activation window slots
  // (1x1 layers, with few weight stages per chunk, want more of them in
  // flight; convolutions reuse one window for all taps) and weight stages.
  auto plan = [&](int mh) {
    pl.win_rows = kBlockM * mh + (mx - mn);
    pl.a_win_bytes = static_cast<uint32_t>(pl.planes * pl.win_rows * 16);
    pl.a_slot_bytes = pl.a_win_bytes;
    pl.m_tiles = (d.rows + kBlockM * mh - 1) / (kBlockM * mh);
    pl.n_tiles = d.cout / bn;
    return chooseSlots(pl.a_win_bytes, pl.b_stage_bytes, pl.stages_per_chunk, &pl.a_slots, &pl.b_stages);
  };
  // CTA pairs over two SMs when there are pair tiles for every pair of SMs:
  // 256-channel tiles with 256-row pair tiles (one row block per CTA), and
  // 64- or 128-channel layers with 512-row pair tiles (two row blocks per CTA,
  // two M=256 MMAs per K step, like the single-CTA 256-row tiles, with half
  // the weight tile staged per SM and one issuing thread for both SMs).
  // Windows of up to 4 x 128 rows, one lane per row-run box.
  const int kprime = pl.n_chunks * d.taps * pl.cw;
  auto s = static_cast<cudaStream_t>(stream);
  const int pair_mh = bn == 256 ? 1 : 2;
  const int pair_planes = pl.cw * esize / 16;
  const int pair_boxes = (pair_mh * kBlockM + (mx - mn) + 127) / 128;  // row-run boxes per window plane
  const bool withhold = g_withhold_loads.load();
  if (!withhold && g_cta_pairs.load() && (bn == 256 || (bn <= 128 && d.cout == bn)) && pair_boxes <= 4 &&
      (pair_boxes == 1 || pair_boxes * pair_planes <= 32)) {
    // For 1x1 layers the weight order does not depend on the chunk width
    // (k' = channel), so wider windows (fewer activation barriers per MMA) are
    // free to choose; the widest that keeps the pipeline as deep is taken.
    // Dense 16-bit outputs (the transformer linears: SAME layout, every row
    // valid) leave the epilogue as TMA bulk stores of staged 32-column chunks.
    const bool tma_store = g_tma_store.load() && esize == 2 && bn == 256 && d.dst_mode == FPK_DST_SAME &&
                           d.grid_w == 1 && d.valid_w >= 1 && d.valid_h >= d.img_rows;
    const size_t stage_reserve = tma_store ? kOutStageBytes + 1024 : 0;
    Plan pp = pl;
    pp.win_rows = pair_mh * kBlockM + (mx - mn);
    pp.b_stage_bytes = static_cast<uint32_t>(bn / 2) * 128u;
    pp.m_tiles = (d.rows + 2 * pair_mh * kBlockM - 1) / (2 * pair_mh * kBlockM);
    pp.n_tiles = d.cout / bn;
    bool planned = false;
    int best_depth = 0;
    for (int cw = pl.cw; cw <= (d.taps == 1 ? 4 * stage_elems : pl.cw) && cw <= d.cin; cw *= 2) {
      if (d.cin % cw != 0) continue;
      Plan c = pp;
      c.cw = cw;
      c.planes = cw * esize / 16;
      c.n_chunks = d.cin / cw;
      c.stages_per_chunk = d.taps * cw / stage_elems;
      if (c.stages_per_chunk > kMaxStagesPerChunk) continue;
      // Bytes moved per window, and its shared-memory footprint: every TMA
      // destination (a plane, or its boxes past row 128) starts on 128 bytes.
      if (c.win_rows > 128 && ((c.win_rows + 127) / 128) * c.planes > 32) continue;  // one lane per box
      c.a_win_bytes = static_cast<uint32_t>(c.planes * c.win_rows * 16);
      c.a_plane_pitch = c.win_rows <= 128 ? static_cast<uint32_t>(c.win_rows * 16)
                                          : (static_cast<uint32_t>(c.win_rows * 16) + 127u) & ~127u;
      c.a_slot_bytes = (static_cast<uint32_t>(c.planes) * c.a_plane_pitch + 1023u) & ~1023u;
      if (!chooseSlots(c.a_slot_bytes, c.b_stage_bytes, c.stages_per_chunk, &c.a_slots, &c.b_stages, stage_reserve)) {
        continue;
      }
      const int depth = c.a_slots * c.stages_per_chunk < c.b_stages ? c.a_slots * c.stages_per_chunk : c.b_stages;
      if (depth >= best_depth) {
        best_depth = depth;
        pp = c;
        planned = true;
      }
    }
    if (planned && pp.m_tiles * pp.n_tiles >= numSms() / 2) {
      size_t smem = 1024 + static_cast<size_t>(pp.b_stages) * pp.b_stage_bytes +
                    static_cast<size_t>(pp.a_slots) * pp.a_slot_bytes + sizeof(Smem);
      pp.tma_store = tma_store ? 1 : 0;
      pp.stage_off = 0;
      if (tma_store) {
        pp.stage_off = static_cast<uint32_t>((smem - 1024 + 1023) & ~static_cast<size_t>(1023));
        smem = 1024 + pp.stage_off + kOutStageBytes;
      }
      CUtensorMap map_w, map_a;
      if (makeWeightMap(d, kprime, bn / 2, &map_w) != 0) return 1;
      CUtensorMap map_out = map_w;  // unused unless tma_store
      if (tma_store && makePlanarRowsMap(d.dst, d.rows, d.cout / 8, d.dst_plane_stride, 32, 4, &map_out,
                                         "fpk_gemm (output)") != 0) {
        return 1;
      }
      CUtensorMap map_a_tail;
      const int total_planes = d.cin * esize / 16;
      if (pp.win_rows <= 128) {
        if (makePlanarRowsMap(d.a, d.rows, total_planes, d.a_plane_stride, pp.win_rows, pp.planes, &map_a,
                              "fpk_gemm") != 0) {
          return 1;
        }
        map_a_tail = map_a;
      } else {
        const int tail_rows = (pp.win_rows & 127) != 0 ? (pp.win_rows & 127) : 128;
        if (makePlanarRowsMap(d.a, d.rows, total_planes, d.a_plane_stride, 128, 1, &map_a, "fpk_gemm") != 0 ||
            makePlanarRowsMap(d.a, d.rows, total_planes, d.a_plane_stride, tail_rows, 1, &map_a_tail, "fpk_gemm") != 0) {
          return 1;
        }
      }
      switch (d.dtype) {
        case FPK_DTYPE_BF16:
          return bn == 256   ? launchPair<__nv_bfloat16, 256, 1>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s)
                 : bn == 128 ? launchPair<__nv_bfloat16, 128, 2>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s)
                             : launchPair<__nv_bfloat16, 64, 2>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s);
        case FPK_DTYPE_F32:
        case FPK_DTYPE_F32_EXACT:
          return bn == 256   ? launchPair<float, 256, 1>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s)
                 : bn == 128 ? launchPair<float, 128, 2>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s)
                             : launchPair<float, 64, 2>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s);
        default:
          return bn == 256   ? launchPair<__half, 256, 1>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s)
                 : bn == 128 ? launchPair<__half, 128, 2>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s)
                             : launchPair<__half, 64, 2>(d, pp, map_w, map_a, map_a_tail, map_out, smem, s);
      }
    }
  }
  // Narrow layers (BN <= 128) take 256-row tiles when there are enough rows
  // to keep every SM busy.
  int mh = 1;
  // 1x1 layers (linears) with 256-column tiles take 256-row tiles too (one
  // accumulator buffer): every activation window then feeds two MMAs per
  // weight stage, which their per-stage copies otherwise saturate shared
  // memory with.
  const bool wide_linear = bn == 256 && d.taps == 1;
  if ((bn <= 128 || wide_linear) && (d.rows + kBlockM - 1) / kBlockM >= 2 * numSms() && plan(2)) {
    mh = 2;
  } else if (!plan(1)) {
    return fail("fpk_gemm: activation window too large for shared memory");
  }
  // Split K when the output tiles fill less than half of the GPU (small
  // batches, e.g. tracking one hypothesis) and the caller gave scratch: up to
  // 8 chunk ranges per tile (the reduce kernel adds at most 8 partials), at
  // most one CTA per SM in all.
  if (mh == 1 && d.splitk_ws != nullptr && pl.n_chunks >= 2) {
    const int tiles = pl.m_tiles * pl.n_tiles;
    int ks = tiles * 2 <= numSms() ? numSms() / tiles : 1;
    ks = ks < pl.n_chunks ? ks : pl.n_chunks;
    ks = ks < kEpilogueWarps ? ks : kEpilogueWarps;
    while (ks > 1 && static_cast<long long>(tiles) * ks * bn * kBlockM * 4 > d.splitk_ws_bytes) --ks;
    if (ks > 1 && reinterpret_cast<uintptr_t>(d.splitk_ws) % 16 == 0) pl.k_splits = ks;
  }
  pl.withhold_loads = withhold ? 1 : 0;
  const size_t smem = 1024 + static_cast<size_t>(pl.b_stages) * pl.b_stage_bytes +
                      static_cast<size_t>(pl.a_slots) * pl.a_win_bytes + sizeof(Smem);
  CUtensorMap map;
  if (makeWeightMap(d, kprime, bn, &map) != 0) return 1;
  switch (d.dtype) {
    case FPK_DTYPE_BF16:
      return launchShape<__nv_bfloat16>(d, pl, map, smem, s, bn, mh);
    case FPK_DTYPE_F32:
    case FPK_DTYPE_F32_EXACT:
      return launchShape<float>(d, pl, map, smem, s, bn, mh);
    default:
      return launchShape<__half>(d, pl, map, smem, s, bn, mh);
  }
}

extern "C" int fpk_gemm_set_cta_pairs(int enable) {
  return fpb::gemm::g_cta_pairs.exchange(enable != 0) ? 1 : 0;
}

extern "C" int fpk_gemm_set_tma_store(int enable) {
  return fpb::gemm::g_tma_store.exchange(enable != 0) ? 1 : 0;
}

extern "C" int fpk_gemm_test_withhold_loads(int enable) {
  return fpb::gemm::g_withhold_loads.exchange(enable != 0) ? 1 : 0;
}

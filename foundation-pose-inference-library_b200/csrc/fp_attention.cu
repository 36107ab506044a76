// Fused self-attention on tcgen05 tensor cores (sm_100a) for the RefineNet /
// ScoreNet transformer layers: softmax(Q K^T / sqrt(128)) V for 4 heads of
// 128 channels over a sequence of 400 tokens, reference network
// RefineNet/ScoreNet nn.TransformerEncoderLayer (batch_first, nhead=4).
//
// One CTA per (query tile, layer * head, sequence). A query tile has up to 128
// rows (TMEM lanes); keys stream in blocks of 64. Warp roles:
//   warp 0     producer: one 2-D TMA tile load per Q tile and per K / V key
//              block from the KP8 planar activations ([plane of 8 channels]
//              [row][16 B]) straight into the no-swizzle core-matrix layout
//              [plane][row][16 B] the tensor core reads (per-plane bulk copies,
//              16 per block, could not be issued as fast as blocks were
//              consumed); key blocks are requested one block ahead of value
//              blocks, three in flight.
//   warp 1     MMA issuer (one lane) + TMEM owner:
//                S_b = Q K_b^T   (M=128, N=64, K=128; A, B K-major)   -> TMEM
//                O  += P_b V_b   (M=128, N=128, K=64; A = P from TMEM,
//                                 B = V MN-major from shared memory)  -> TMEM
//              S is double-buffered so S_{b+1} runs while block b is in the
//              softmax; a buffer is reused once the PV product that read its
//              P has completed.
//   warps 2-5  softmax, one query row per thread: one tcgen05.ld of the row's
//              64 scores, running max / sum in the log2 domain, P = 2^(s - m)
//              packed as fp16/bf16 pairs and stored (tcgen05.st) over the first
//              32 columns of the same S buffer. O is rescaled in TMEM only when
//              a row's maximum grows by more than 8 (a factor of 256), which
//              keeps P below 256 and the result exact; at the end O / l is
//              written back to KP8.
// fp16/bf16 run kind::f16 with 96 KB of shared memory and 256 TMEM columns
// per CTA, so two CTAs share an SM and overlap each other's loads, softmax and
// MMAs; fp32 activations run kind::tf32 (TF32 math) with 192 KB, one CTA. All mbarrier waits are
// bounded (fp_tc.cuh) and report through AttnArgs::error_flag.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <atomic>
#include <cstdint>
#include <string>
#include <type_traits>

#include "fp_launch.hpp"
#include "fp_net_kernels.cuh"
#include "fp_profile.hpp"
#include "fp_tc.cuh"
#include "fpk.h"

namespace fpb {
namespace attn {

using namespace fpb::tc;

constexpr int kRows = 128;                 // query rows per tile = TMEM lanes
constexpr int kKeys = 64;                  // keys per block
constexpr int kHeadDim = 128;

// Per element type: 16-byte records hold 8 (fp16/bf16) or 4 (fp32) channels;
// every MMA K step reads 32 bytes (two records) of each row: K=16 under
// kind::f16, K=8 under kind::tf32.
template <typename T>
struct Geo {
  static constexpr bool kTf32 = std::is_same<T, float>::value;
  static constexpr int kPerRecord = 16 / static_cast<int>(sizeof(T));
  static constexpr int kPlanes = kHeadDim / kPerRecord;            // 16 or 32
  static constexpr uint32_t kQBytes = kPlanes * kRows * 16;        // 32 or 64 KB
  static constexpr uint32_t kKVBytes = kPlanes * kKeys * 16;       // 16 or 32 KB
  static constexpr int kStepKeys = 32 / static_cast<int>(sizeof(T));  // keys per PV K step
  // TF32 takes MN-major operands only in the 32-byte-atom 128B swizzle, so
  // fp32 V blocks are transposed in shared memory by two extra warps into a
  // K-major [4-key plane][channel][16 B] tile, from a staging copy whose
  // planes are padded by 16 bytes (conflict-free column reads). P is kept in
  // shared memory too, as a K-major [4-key plane][row][16 B] tile.
  static constexpr int kThreads = kTf32 ? 256 : 192;
  // Key blocks in flight: three for 16-bit (a block arrives from DRAM about two
  // block-times after it is requested), two for fp32 (no shared memory left).
  static constexpr int kKSlots = kTf32 ? 2 : 3;
  static constexpr uint32_t kVRawPlane = kKeys * 16 + (kTf32 ? 16 : 0);
  static constexpr uint32_t kVBytes = kTf32 ? kPlanes * kVRawPlane : 2 * kKVBytes;
  static constexpr uint32_t kVTBytes = kTf32 ? kKVBytes : 0;
  static constexpr uint32_t kPBytes = kTf32 ? (kKeys / kPerRecord) * kRows * 16 : 0;
  static constexpr size_t kSmem = 128 + kQBytes + kKSlots * kKVBytes + kVBytes + kVTBytes + kPBytes + 256;
  static constexpr int kMinBlocks = kTf32 ? 1 : 2;
  static constexpr uint32_t fmt() { return kTf32 ? 2u : (std::is_same<T, __nv_bfloat16>::value ? 1u : 0u); }
};
constexpr uint32_t kTmemCols = 256;        // S[2] (2 x 64) + O (128)
constexpr uint32_t kOCol = 2 * kKeys;
constexpr float kRescaleLog2 = 8.0f;

struct Bars {
  uint64_t q_full;
  uint64_t k_full[3], k_empty[3];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full, p_free;  // P_b ready / PV_b complete
  uint64_t vt_full, vt_empty;  // fp32: transposed V tile ready / consumed
  uint64_t o_done;
  uint32_t tmem_base;
};

static_assert(sizeof(Bars) <= 256, "barrier block");

// Instruction descriptor: fp32 accumulate, A K-major, B K- or MN-major.
__host__ __device__ constexpr uint32_t idesc(uint32_t fmt, int n, bool b_mn_major) {
  return (1u << 4) | (fmt << 7) | (fmt << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(kRows >> 4) << 24);
}

// MMAs issued by one elected lane of the (converged) issuing warp.
template <typename T>
__device__ __forceinline__ void mmaSS(uint32_t d, uint64_t a, uint64_t b, uint32_t id, uint32_t acc) {
  if constexpr (Geo<T>::kTf32) {
    tcMmaTf32Elect(d, a, b, id, acc);
  } else {
    tcMmaElect(d, a, b, id, acc);
  }
}

template <typename T>
__device__ __forceinline__ void mmaTS(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t id, uint32_t acc) {
  if constexpr (Geo<T>::kTf32) {
    tcMmaTf32TmemAElect(d, a_tmem, b, id, acc);
  } else {
    tcMmaTmemAElect(d, a_tmem, b, id, acc);
  }
}

// 2^x with the MUFU ex2 instruction (flush-to-zero, ~2 ulp); 2^-inf = 0.
__device__ __forceinline__ float exp2Approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

template <typename T>
__global__ void __launch_bounds__(Geo<T>::kThreads, Geo<T>::kMinBlocks)
    attentionTcKernel(const net::AttnArgs a, const __grid_constant__ CUtensorMap q_map,
                      const __grid_constant__ CUtensorMap kv_map) {
  using G = Geo<T>;
  constexpr int kPlanes = G::kPlanes;
  constexpr uint32_t kQBytes = G::kQBytes;
  constexpr uint32_t kKVBytes = G::kKVBytes;
  pdlTrigger();
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  unsigned char* q_s = base;
  unsigned char* k_s = q_s + kQBytes;           // [kKSlots][planes][64 keys][16 B]
  unsigned char* v_s = k_s + G::kKSlots * kKVBytes;  // [2][planes][64 keys][16 B]; fp32: padded staging
  unsigned char* vt_s = v_s + G::kVBytes;       // fp32 only: [16 key planes][128 ch][16 B]
  unsigned char* p_s = vt_s + G::kVTBytes;      // fp32 only: [16 key planes][128 rows][16 B]
  Bars* bars = reinterpret_cast<Bars*>(p_s + G::kPBytes);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  int* err = a.error_flag;

  const int q_tiles = gridDim.x;
  const int q_rows = (a.seq_len + q_tiles - 1) / q_tiles;  // <= 128 by construction
  const int q0 = blockIdx.x * q_rows;
  const int valid_q = min(q_rows, a.seq_len - q0);
  const int layer = blockIdx.y / a.heads;
  const int head = blockIdx.y - layer * a.heads;
  const long long row_base = static_cast<long long>(blockIdx.z) * a.seq_len;
  const int n_blocks = (a.seq_len + kKeys - 1) / kKeys;

  if (threadIdx.x == 0) {
    mbarInit(&bars->q_full, 1);
    for (int i = 0; i < G::kKSlots; ++i) {
      mbarInit(&bars->k_full[i], 1);
      mbarInit(&bars->k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbarInit(&bars->v_full[i], 1);
      mbarInit(&bars->v_empty[i], G::kTf32 ? 2 : 1);
      mbarInit(&bars->s_full[i], 1);
      mbarInit(&bars->s_free[i], 1);
    }
    mbarInit(&bars->p_full, 4);
    mbarInit(&bars->p_free, 1);
    mbarInit(&bars->o_done, 1);
    mbarInit(&bars->vt_full, 2);
    mbarInit(&bars->vt_empty, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smemU32(&bars->tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  __syncthreads();
  tcFenceAfter();
  pdlWait();  // the QKV projection is complete from here on
  const uint32_t tmem = bars->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      const int qp = layer * a.qkv_layer_planes + a.q_plane + head * kPlanes;
      const int kp = layer * a.qkv_layer_planes + a.k_plane + head * kPlanes;
      const int vp = layer * a.qkv_layer_planes + a.v_plane + head * kPlanes;
      // Rows past the sequence (the tile tail, the last key block) read the
      // next sequence or the buffer's zero guard rows: finite values whose
      // scores are masked and whose outputs are not stored.
      // One tile load per operand block ({rows x 16 B, planes} boxes land as
      // [plane][row][16 B]); rows past the buffer read as zeros.
      mbarExpectTx(&bars->q_full, kQBytes);
      tmaLoad2d(q_s, &q_map, static_cast<int>(2 * (row_base + q0)), qp, &bars->q_full);
      bool ok = true;
      int k_issued = 0, v_issued = 0;
      // Key block b goes to slot b % kKSlots once S_{b - kKSlots} has read it;
      // key blocks are requested one block ahead of value blocks, so a key
      // load never waits behind a value slot.
      auto issueK = [&](int b) -> bool {
        const int slot = b % G::kKSlots;
        if (b >= G::kKSlots && !waitBar(&bars->k_empty[slot], ((b / G::kKSlots) - 1) & 1, err, 21)) return false;
        const long long r0 = row_base + static_cast<long long>(b) * kKeys;
        mbarExpectTx(&bars->k_full[slot], kKVBytes);
        tmaLoad2d(k_s + slot * kKVBytes, &kv_map, static_cast<int>(2 * r0), kp, &bars->k_full[slot]);
        k_issued = b + 1;
        return true;
      };
      ok = issueK(0);
      for (int b = 0; b < n_blocks && ok; ++b) {
        if (b + 1 < n_blocks) ok = issueK(b + 1);
        if (!ok) break;
        // V: double-buffered (16-bit), or one staging buffer (fp32) that the
        // transpose warps release.
        const int slot = b & 1;
        const long long r0 = row_base + static_cast<long long>(b) * kKeys;
        const int vslot = G::kTf32 ? 0 : slot;
        if (G::kTf32 ? b >= 1 : b >= 2) {
          ok = waitBar(&bars->v_empty[vslot], G::kTf32 ? ((b - 1) & 1) : (((b >> 1) - 1) & 1), err, 22);
        }
        if (!ok) break;
        mbarExpectTx(&bars->v_full[vslot], kKVBytes);
        if constexpr (G::kTf32) {
          // fp32: per-plane copies into the padded staging planes.
          for (int p = 0; p < kPlanes; ++p) {
            bulkCopy(v_s + p * G::kVRawPlane, a.qkv + static_cast<long long>(vp + p) * a.qkv_plane_stride + r0 * 16,
                     kKeys * 16, &bars->v_full[vslot]);
          }
        } else {
          tmaLoad2d(v_s + slot * kKVBytes, &kv_map, static_cast<int>(2 * r0), vp, &bars->v_full[vslot]);
        }
        v_issued = b + 1;
      }
      // Drain: every copy armed above lands before the CTA may exit.
      drainBar(&bars->q_full, 0);
      for (int b = k_issued > G::kKSlots ? k_issued - G::kKSlots : 0; b < k_issued; ++b) {
        drainBar(&bars->k_full[b % G::kKSlots], (b / G::kKSlots) & 1);
      }
      // fp32 stages V through one buffer: only the last block can still be in
      // flight, and an earlier block's parity already names a later phase of
      // the same barrier (waiting on it would only end at the timeout).
      const int v_in_flight = G::kTf32 ? 1 : 2;
      for (int b = v_issued > v_in_flight ? v_issued - v_in_flight : 0; b < v_issued; ++b) {
        if (G::kTf32) {
          drainBar(&bars->v_full[0], b & 1);
        } else {
          drainBar(&bars->v_full[b & 1], (b >> 1) & 1);
        }
      }
    }
  } else if (warp == 1) {
    {
      // ---------------- MMA issuer ----------------
      // The whole warp runs the loop (warp-uniform descriptors); an elected
      // lane issues each tcgen05 instruction.
      // PV: V as an MN-major B operand (16-bit), or the transposed K-major tile (fp32).
      const uint32_t idesc_o = idesc(G::fmt(), kHeadDim, !G::kTf32);
      const uint32_t q_addr = smemU32(q_s);
      const uint32_t k_addr = smemU32(k_s);
      const uint32_t v_addr = smemU32(v_s);
      bool ok = warpWaitBar(&bars->q_full, 0, err, 23);
      tcFenceAfter();
      for (int b = 0; b <= n_blocks && ok; ++b) {
        if (b < n_blocks) {
          const int slot = b & 1;               // S buffer
          const int kslot = b % G::kKSlots;     // key block
          ok = warpWaitBar(&bars->k_full[kslot], (b / G::kKSlots) & 1, err, 24);
          if (ok && b >= 2) ok = warpWaitBar(&bars->s_free[slot], ((b >> 1) - 1) & 1, err, 25);
          if (!ok) break;
          tcFenceAfter();
          const int keys = min(kKeys, a.seq_len - b * kKeys);
          const int n = (keys + 15) & ~15;
          const uint32_t idesc_s = idesc(G::fmt(), n, false);
          const uint32_t d = tmem + static_cast<uint32_t>(slot * kKeys);
#pragma unroll
          for (int ks = 0; ks < kPlanes / 2; ++ks) {
            // 32 bytes of head channels = two planes per K step.
            const uint64_t ad = smemDesc(q_addr + ks * 2 * (kRows * 16), kRows * 16, 128, kLayoutNone);
            const uint64_t bd = smemDesc(k_addr + kslot * kKVBytes + ks * 2 * (kKeys * 16), kKeys * 16,
                                         128, kLayoutNone);
            mmaSS<T>(d, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
          }
          tcCommitElect(&bars->s_full[slot]);
          tcCommitElect(&bars->k_empty[kslot]);
        }
        if (b >= 1) {
          const int j = b - 1;
          const int slot = j & 1;
          ok = warpWaitBar(&bars->p_full, j & 1, err, 26);
          if (ok) {
            ok = G::kTf32 ? warpWaitBar(&bars->vt_full, j & 1, err, 27)
                          : warpWaitBar(&bars->v_full[slot], (j >> 1) & 1, err, 27);
          }
          if (!ok) break;
          tcFenceAfter();
          const int keys = min(kKeys, a.seq_len - j * kKeys);
          const int steps = (keys + G::kStepKeys - 1) / G::kStepKeys;
          for (int ks = 0; ks < steps; ++ks) {
            // P: A operand in TMEM, one K step = 8 columns (16 keys packed in
            // pairs, or 8 fp32 keys). V: MN-major B, 8-key core matrices 128 B
            // apart (LBO), channel planes kKeys*16 bytes apart (SBO).
            if constexpr (G::kTf32) {
              // 8 keys = two 4-key planes per K step, for P (A) and V^T (B).
              const uint64_t ad = smemDesc(smemU32(p_s) + ks * 2 * (kRows * 16), kRows * 16, 128, kLayoutNone);
              const uint64_t bd = smemDesc(smemU32(vt_s) + ks * 2 * (kHeadDim * 16), kHeadDim * 16, 128,
                                           kLayoutNone);
              mmaSS<T>(tmem + kOCol, ad, bd, idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
            } else {
              const uint64_t bd = smemDesc(v_addr + slot * kKVBytes + ks * G::kStepKeys * 16, 128,
                                           kKeys * 16, kLayoutNone);
              const uint32_t at = tmem + static_cast<uint32_t>(slot * kKeys + ks * 8);
              mmaTS<T>(tmem + kOCol, at, bd, idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
            }
          }
          tcCommitElect(&bars->p_free);
          tcCommitElect(G::kTf32 ? &bars->vt_empty : &bars->v_empty[slot]);
          tcCommitElect(&bars->s_free[slot]);
        }
      }
      tcCommitElect(&bars->o_done);
      if (lane == 0) drainBar(&bars->o_done, 0);
      __syncwarp();
    }
  } else if (warp < 6) {
    // ---------------- softmax + output (warps 2..5) ----------------
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16);
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int b = 0; b < n_blocks && ok; ++b) {
      const int slot = b & 1;
      ok = waitBar(&bars->s_full[slot], (b >> 1) & 1, err, 28);
      if (!ok) break;
      tcFenceAfter();
      const int keys = min(kKeys, a.seq_len - b * kKeys);
      // One TMEM read of the row's 64 scores (two 32-column loads, one wait).
      uint32_t sv[kKeys];
      FPB_TMEM_LD32(lane_base + slot * kKeys, sv);
      FPB_TMEM_LD32(lane_base + slot * kKeys + 32, (sv + 32));
      tmemWaitLd();
      if (keys < kKeys) {
        // Last block: keys past the sequence contribute nothing.
#pragma unroll
        for (int e = 0; e < kKeys; ++e) {
          if (e >= keys) sv[e] = __float_as_uint(-INFINITY);
        }
      }
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < kKeys; ++e) mx = fmaxf(mx, __uint_as_float(sv[e]));
      const float mb = mx * a.scale_log2;  // scale_log2 > 0 commutes with max
      const float m_new = fmaxf(m, mb);
      if (b == 0) {
        m = m_new;
      } else {
        const bool grow = m_new > m + kRescaleLog2;
        if (__any_sync(0xffffffffu, grow)) {
          // O holds blocks < b once PV_{b-1} has completed.
          ok = waitBar(&bars->p_free, (b - 1) & 1, err, 29);
          if (!ok) break;
          tcFenceAfter();
          const float f = grow ? exp2Approx(m - m_new) : 1.0f;
#pragma unroll 1
          for (int c = 0; c < 128; c += 32) {
            uint32_t ov[32];
            FPB_TMEM_LD32(lane_base + kOCol + c, ov);
            tmemWaitLd();
#pragma unroll
            for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * f);
            FPB_TMEM_ST32(lane_base + kOCol + c, ov);
          }
          tmemStoreWait();
          if (grow) {
            l *= f;
            m = m_new;
          }
        }
      }
      // P = 2^(s * scale - m) (masked keys give 2^-inf = 0) over this S
      // buffer: the PV product's A operand (16-bit pairs in the first 32
      // columns, or fp32 in place).
      const float neg_m = -m;
      if constexpr (G::kTf32) {
        // The single P buffer is free once PV_{b-1} has completed.
        if (b >= 1) {
          ok = waitBar(&bars->p_free, (b - 1) & 1, err, 31);
          if (!ok) break;
        }
#pragma unroll
        for (int e = 0; e < kKeys; e += 4) {
          float4 w;
          w.x = exp2Approx(fmaf(__uint_as_float(sv[e + 0]), a.scale_log2, neg_m));
          w.y = exp2Approx(fmaf(__uint_as_float(sv[e + 1]), a.scale_log2, neg_m));
          w.z = exp2Approx(fmaf(__uint_as_float(sv[e + 2]), a.scale_log2, neg_m));
          w.w = exp2Approx(fmaf(__uint_as_float(sv[e + 3]), a.scale_log2, neg_m));
          l += (w.x + w.y) + (w.z + w.w);
          *reinterpret_cast<float4*>(p_s + (e >> 2) * (kRows * 16) + r * 16) =
              make_float4(tf32Round(w.x), tf32Round(w.y), tf32Round(w.z), tf32Round(w.w));
        }
        fenceProxyAsyncSmem();
      } else {
        uint32_t pk[kKeys / 2];
#pragma unroll
        for (int e = 0; e < kKeys; e += 2) {
          const float p0 = exp2Approx(fmaf(__uint_as_float(sv[e]), a.scale_log2, neg_m));
          const float p1 = exp2Approx(fmaf(__uint_as_float(sv[e + 1]), a.scale_log2, neg_m));
          l += p0 + p1;
          pk[e >> 1] = pack2<T>(p0, p1);
        }
        FPB_TMEM_ST32(lane_base + slot * kKeys, pk);
      }
      tmemStoreWait();
      tcFenceBefore();
      __syncwarp();
      if (lane == 0) mbarArrive(&bars->p_full);
    }
    if (ok) ok = waitBar(&bars->o_done, 0, err, 30);
    // The MMA warp also signals o_done when it gave up part-way (it drains on
    // that barrier): after any reported error O is not stored.
    if (ok && *reinterpret_cast<volatile int*>(err) != 0) ok = false;
    if (ok) {
      tcFenceAfter();
      const float inv = 1.0f / l;
      const int op = layer * a.out_layer_planes + head * kPlanes;
      const bool store = r < valid_q;
      unsigned char* out = a.out + (row_base + q0 + r) * 16;
#pragma unroll 1
      for (int c = 0; c < 128; c += 32) {
        uint32_t ov[32];
        FPB_TMEM_LD32(lane_base + kOCol + c, ov);
        tmemWaitLd();
        if (store) {
          if constexpr (G::kTf32) {
#pragma unroll
            for (int g = 0; g < 8; ++g) {
              const float4 w = make_float4(tf32Round(__uint_as_float(ov[g * 4 + 0]) * inv),
                                           tf32Round(__uint_as_float(ov[g * 4 + 1]) * inv),
                                           tf32Round(__uint_as_float(ov[g * 4 + 2]) * inv),
                                           tf32Round(__uint_as_float(ov[g * 4 + 3]) * inv));
              *reinterpret_cast<float4*>(out + static_cast<long long>(op + (c >> 2) + g) * a.out_plane_stride) = w;
            }
          } else {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 w;
              w.x = pack2<T>(__uint_as_float(ov[g * 8 + 0]) * inv, __uint_as_float(ov[g * 8 + 1]) * inv);
              w.y = pack2<T>(__uint_as_float(ov[g * 8 + 2]) * inv, __uint_as_float(ov[g * 8 + 3]) * inv);
              w.z = pack2<T>(__uint_as_float(ov[g * 8 + 4]) * inv, __uint_as_float(ov[g * 8 + 5]) * inv);
              w.w = pack2<T>(__uint_as_float(ov[g * 8 + 6]) * inv, __uint_as_float(ov[g * 8 + 7]) * inv);
              *reinterpret_cast<uint4*>(out + static_cast<long long>(op + (c >> 3) + g) * a.out_plane_stride) = w;
            }
          }
        }
      }
    }
    tcFenceBefore();
  } else if constexpr (G::kTf32) {
    // ---------------- V transpose (fp32 only, warps 6..7) ----------------
    // staging [ch plane][key][4 ch] -> V^T [key plane][ch][4 keys].
    const int t = threadIdx.x - 192;  // 0..63
    bool ok = true;
    for (int b = 0; b < n_blocks && ok; ++b) {
      ok = waitBar(&bars->v_full[0], b & 1, err, 32);
      if (ok && b >= 1) ok = waitBar(&bars->vt_empty, (b - 1) & 1, err, 33);
      if (!ok) break;
      tcFenceAfter();
      for (int rec = t; rec < (kKeys / 4) * kHeadDim; rec += 64) {
        const int kp = rec / kHeadDim;
        const int ch = rec - kp * kHeadDim;
        const float* src = reinterpret_cast<const float*>(v_s + (ch >> 2) * G::kVRawPlane + kp * 64) + (ch & 3);
        *reinterpret_cast<float4*>(vt_s + kp * (kHeadDim * 16) + ch * 16) =
            make_float4(src[0], src[4], src[8], src[12]);
      }
      fenceProxyAsyncSmem();
      __syncwarp();
      if ((threadIdx.x & 31) == 0) {
        mbarArrive(&bars->v_empty[0]);
        mbarArrive(&bars->vt_full);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tcFenceAfter();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <typename T>
cudaError_t launch(const net::AttnArgs& a, int layers, int n_seq, cudaStream_t s) {
  static DeviceOnce smem_attr;
  const cudaError_t ae = smem_attr.run([] {
    return cudaFuncSetAttribute(attentionTcKernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                static_cast<int>(Geo<T>::kSmem));
  });
  if (ae != cudaSuccess) return ae;
  const int q_tiles = (a.seq_len + kRows - 1) / kRows;
  // Maps over the whole qkv buffer: every plane of every layer, every row of
  // every sequence; the kernel indexes blocks by (row, first plane).
  CUtensorMap q_map, kv_map;
  const long long rows = static_cast<long long>(n_seq) * a.seq_len;
  const int planes = layers * a.qkv_layer_planes;
  if (makePlanarRowsMap(a.qkv, rows, planes, a.qkv_plane_stride, kRows, Geo<T>::kPlanes, &q_map, "fpk_attention") != 0 ||
      makePlanarRowsMap(a.qkv, rows, planes, a.qkv_plane_stride, kKeys, Geo<T>::kPlanes, &kv_map, "fpk_attention") != 0) {
    return cudaErrorInvalidValue;
  }
  prof::countLaunch(prof::kAttention);
  return launchPdl(attentionTcKernel<T>, dim3(q_tiles, layers * a.heads, n_seq), dim3(Geo<T>::kThreads), Geo<T>::kSmem,
                   s, a, q_map, kv_map);
}

}  // namespace attn

namespace net {

cudaError_t launchAttentionTc(const AttnArgs& a, int layers, int n_seq, int dtype, cudaStream_t s) {
  if (a.seq_len <= 0 || a.error_flag == nullptr) return cudaErrorInvalidValue;
  switch (dtype) {
    case FPK_DTYPE_BF16:
      return attn::launch<__nv_bfloat16>(a, layers, n_seq, s);
    case FPK_DTYPE_F32:
      return attn::launch<float>(a, layers, n_seq, s);
    case FPK_DTYPE_F32_EXACT:
      return launchAttentionExact(a, layers, n_seq, s);
    default:
      return attn::launch<__half>(a, layers, n_seq, s);
  }
}

}  // namespace net
}  // namespace fpb

namespace fpb {
int fail(const std::string& msg);
int checkLaunch(const char* what);
}  // namespace fpb

extern "C" int fpk_attention(const void* qkv, long long qkv_plane_stride, int qkv_layer_channels,
                             int q_channel, int k_channel, int v_channel, void* out,
                             long long out_plane_stride, int out_layer_channels, int layers, int heads,
                             int seq_len, int n_seq, int dtype, int* error_flag, void* stream) {
  if (qkv == nullptr || out == nullptr || error_flag == nullptr) return fpb::fail("fpk_attention: null pointer");
  if (dtype != FPK_DTYPE_F16 && dtype != FPK_DTYPE_BF16 && dtype != FPK_DTYPE_F32 && dtype != FPK_DTYPE_F32_EXACT) {
    return fpb::fail("fpk_attention: dtype must be f16, bf16, f32 or f32-exact");
  }
  const int per = (dtype == FPK_DTYPE_F32 || dtype == FPK_DTYPE_F32_EXACT) ? 4 : 8;
  if (seq_len <= 0 || n_seq <= 0 || layers <= 0 || heads <= 0 || qkv_layer_channels % per ||
      q_channel % per || k_channel % per || v_channel % per || out_layer_channels % per) {
    return fpb::fail("fpk_attention: bad sizes");
  }
  if (reinterpret_cast<uintptr_t>(qkv) % 16 || reinterpret_cast<uintptr_t>(out) % 16 ||
      qkv_plane_stride % 16 || out_plane_stride % 16) {
    return fpb::fail("fpk_attention: pointers and plane strides must be 16-byte aligned");
  }
  fpb::net::AttnArgs a{};
  a.qkv = static_cast<const unsigned char*>(qkv);
  a.qkv_plane_stride = qkv_plane_stride;
  a.qkv_layer_planes = qkv_layer_channels / per;
  a.q_plane = q_channel / per;
  a.k_plane = k_channel / per;
  a.v_plane = v_channel / per;
  a.out = static_cast<unsigned char*>(out);
  a.out_plane_stride = out_plane_stride;
  a.out_layer_planes = out_layer_channels / per;
  a.seq_len = seq_len;
  a.heads = heads;
  a.scale_log2 = 1.4426950408889634f / std::sqrt(128.0f);
  a.error_flag = error_flag;
  const cudaError_t e = fpb::net::launchAttentionTc(a, layers, n_seq, dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fpb::fail(std::string("fpk_attention: ") + cudaGetErrorString(e));
  return 0;
}

// Fused self-attention on tcgen05 tensor cores (sm_100a) for the RefineNet /
// ScoreNet transformer layers: softmax(Q K^T / sqrt(128)) V for 4 heads of
// 128 channels over a sequence of 400 tokens, reference network
// RefineNet/ScoreNet nn.TransformerEncoderLayer (batch_first, nhead=4).
//
// One CTA per (query tile, layer * head, sequence). A query tile has up to 128
// rows (TMEM lanes); keys stream in blocks of 64. Warp roles:
//   warp 0     producer: bulk copies of the Q tile and of K / V key blocks from
//              the KP8 planar activations ([plane of 8 channels][row][16 B])
//              straight into the no-swizzle core-matrix layout
//              [plane][row][16 B] the tensor core reads.
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
// Shared memory 96 KB and 256 TMEM columns per CTA, so two CTAs share an SM
// and overlap each other's loads, softmax and MMAs. All mbarrier waits are
// bounded (fp_tc.cuh) and report through AttnArgs::error_flag.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "fp_net_kernels.cuh"
#include "fp_tc.cuh"

namespace fpb {
namespace attn {

using namespace fpb::tc;

constexpr int kRows = 128;                 // query rows per tile = TMEM lanes
constexpr int kKeys = 64;                  // keys per block
constexpr int kPlanes = 16;                // 128 head channels / 8
constexpr uint32_t kQBytes = kPlanes * kRows * 16;   // 32 KB
constexpr uint32_t kKVBytes = kPlanes * kKeys * 16;  // 16 KB
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;        // S[2] (2 x 64) + O (128)
constexpr uint32_t kOCol = 2 * kKeys;
constexpr float kRescaleLog2 = 8.0f;

struct Bars {
  uint64_t q_full;
  uint64_t k_full[2], k_empty[2];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full, p_free;  // P_b in TMEM ready / PV_b complete
  uint64_t o_done;
  uint32_t tmem_base;
};

constexpr size_t kSmemBytes = 128 + kQBytes + 4 * kKVBytes + sizeof(Bars);

__host__ __device__ constexpr uint32_t idescF16(int n, bool bf16, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) |
         ((b_mn_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(kRows >> 4) << 24);
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
__global__ void __launch_bounds__(kThreads, 2) attentionTcKernel(const net::AttnArgs a) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  unsigned char* base = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  unsigned char* q_s = base;
  unsigned char* k_s = q_s + kQBytes;           // [2][16 planes][64 keys][16 B]
  unsigned char* v_s = k_s + 2 * kKVBytes;      // [2][16 planes][64 keys][16 B]
  Bars* bars = reinterpret_cast<Bars*>(v_s + 2 * kKVBytes);

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
    for (int i = 0; i < 2; ++i) {
      mbarInit(&bars->k_full[i], 1);
      mbarInit(&bars->k_empty[i], 1);
      mbarInit(&bars->v_full[i], 1);
      mbarInit(&bars->v_empty[i], 1);
      mbarInit(&bars->s_full[i], 1);
      mbarInit(&bars->s_free[i], 1);
    }
    mbarInit(&bars->p_full, 4);
    mbarInit(&bars->p_free, 1);
    mbarInit(&bars->o_done, 1);
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
      mbarExpectTx(&bars->q_full, kQBytes);
      for (int p = 0; p < kPlanes; ++p) {
        bulkCopy(q_s + p * (kRows * 16),
                 a.qkv + static_cast<long long>(qp + p) * a.qkv_plane_stride + (row_base + q0) * 16,
                 kRows * 16, &bars->q_full);
      }
      bool ok = true;
      int issued = 0;
      for (int b = 0; b < n_blocks && ok; ++b) {
        const int slot = b & 1;
        const long long r0 = row_base + static_cast<long long>(b) * kKeys;
        if (b >= 2) ok = waitBar(&bars->k_empty[slot], ((b >> 1) - 1) & 1, err, 21);
        if (!ok) break;
        mbarExpectTx(&bars->k_full[slot], kKVBytes);
        for (int p = 0; p < kPlanes; ++p) {
          bulkCopy(k_s + slot * kKVBytes + p * (kKeys * 16),
                   a.qkv + static_cast<long long>(kp + p) * a.qkv_plane_stride + r0 * 16,
                   kKeys * 16, &bars->k_full[slot]);
        }
        if (b >= 2) ok = waitBar(&bars->v_empty[slot], ((b >> 1) - 1) & 1, err, 22);
        if (!ok) {
          issued = 2 * b + 1;
          break;
        }
        mbarExpectTx(&bars->v_full[slot], kKVBytes);
        for (int p = 0; p < kPlanes; ++p) {
          bulkCopy(v_s + slot * kKVBytes + p * (kKeys * 16),
                   a.qkv + static_cast<long long>(vp + p) * a.qkv_plane_stride + r0 * 16,
                   kKeys * 16, &bars->v_full[slot]);
        }
        issued = 2 * b + 2;
      }
      // Drain: every copy armed above lands before the CTA may exit.
      drainBar(&bars->q_full, 0);
      for (int i = issued > 4 ? issued - 4 : 0; i < issued; ++i) {
        const int b = i >> 1;
        drainBar((i & 1) ? &bars->v_full[b & 1] : &bars->k_full[b & 1], (b >> 1) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr bool kBf16 = std::is_same<T, __nv_bfloat16>::value;
      const uint32_t idesc_o = idescF16(128, kBf16, true);
      const uint32_t q_addr = smemU32(q_s);
      const uint32_t k_addr = smemU32(k_s);
      const uint32_t v_addr = smemU32(v_s);
      bool ok = waitBar(&bars->q_full, 0, err, 23);
      tcFenceAfter();
      for (int b = 0; b <= n_blocks && ok; ++b) {
        if (b < n_blocks) {
          const int slot = b & 1;
          ok = waitBar(&bars->k_full[slot], (b >> 1) & 1, err, 24);
          if (ok && b >= 2) ok = waitBar(&bars->s_free[slot], ((b >> 1) - 1) & 1, err, 25);
          if (!ok) break;
          tcFenceAfter();
          const int keys = min(kKeys, a.seq_len - b * kKeys);
          const int n = (keys + 15) & ~15;
          const uint32_t idesc_s = idescF16(n, kBf16, false);
          const uint32_t d = tmem + static_cast<uint32_t>(slot * kKeys);
#pragma unroll
          for (int ks = 0; ks < kPlanes / 2; ++ks) {
            // 16 head channels = two planes per K step.
            const uint64_t ad = smemDesc(q_addr + ks * 2 * (kRows * 16), kRows * 16, 128, kLayoutNone);
            const uint64_t bd = smemDesc(k_addr + slot * kKVBytes + ks * 2 * (kKeys * 16), kKeys * 16,
                                         128, kLayoutNone);
            tcMma(d, ad, bd, idesc_s, ks > 0 ? 1u : 0u);
          }
          tcCommit(&bars->s_full[slot]);
          tcCommit(&bars->k_empty[slot]);
        }
        if (b >= 1) {
          const int j = b - 1;
          const int slot = j & 1;
          ok = waitBar(&bars->p_full, j & 1, err, 26);
          if (ok) ok = waitBar(&bars->v_full[slot], (j >> 1) & 1, err, 27);
          if (!ok) break;
          tcFenceAfter();
          const int keys = min(kKeys, a.seq_len - j * kKeys);
          const int steps = (keys + 15) >> 4;
          for (int ks = 0; ks < steps; ++ks) {
            // P: A operand in TMEM, 16 keys = 8 columns of packed pairs. V:
            // MN-major B, 8-key core matrices 128 B apart (LBO), 8-channel
            // planes kKeys*16 bytes apart (SBO).
            const uint32_t at = tmem + static_cast<uint32_t>(slot * kKeys + ks * 8);
            const uint64_t bd = smemDesc(v_addr + slot * kKVBytes + ks * 16 * 16, 128, kKeys * 16,
                                         kLayoutNone);
            tcMmaTmemA(tmem + kOCol, at, bd, idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
          }
          tcCommit(&bars->p_free);
          tcCommit(&bars->v_empty[slot]);
          tcCommit(&bars->s_free[slot]);
        }
      }
      tcCommit(&bars->o_done);
      drainBar(&bars->o_done, 0);
    }
  } else {
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
      // P = 2^(s * scale - m) (masked keys give 2^-inf = 0), packed in pairs
      // over the first 32 columns of this S buffer: the PV product's A operand.
      const float neg_m = -m;
      uint32_t pk[kKeys / 2];
#pragma unroll
      for (int e = 0; e < kKeys; e += 2) {
        const float p0 = exp2Approx(fmaf(__uint_as_float(sv[e]), a.scale_log2, neg_m));
        const float p1 = exp2Approx(fmaf(__uint_as_float(sv[e + 1]), a.scale_log2, neg_m));
        l += p0 + p1;
        pk[e >> 1] = pack2<T>(p0, p1);
      }
      FPB_TMEM_ST32(lane_base + slot * kKeys, pk);
      tmemStoreWait();
      tcFenceBefore();
      __syncwarp();
      if (lane == 0) mbarArrive(&bars->p_full);
    }
    if (ok) ok = waitBar(&bars->o_done, 0, err, 30);
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
    tcFenceBefore();
  }
  __syncthreads();
  if (warp == 1) {
    tcFenceAfter();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <typename T>
cudaError_t launch(const net::AttnArgs& a, int layers, int n_seq, cudaStream_t s) {
  static int attr_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 31 && !(attr_mask & (1 << dev))) {
    const cudaError_t e = cudaFuncSetAttribute(attentionTcKernel<T>,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    attr_mask |= 1 << dev;
  }
  const int q_tiles = (a.seq_len + kRows - 1) / kRows;
  attentionTcKernel<T><<<dim3(q_tiles, layers * a.heads, n_seq), kThreads, kSmemBytes, s>>>(a);
  return cudaGetLastError();
}

}  // namespace attn

namespace net {

cudaError_t launchAttentionTc(const AttnArgs& a, int layers, int n_seq, bool bf16, cudaStream_t s) {
  if (a.seq_len <= 0 || a.error_flag == nullptr) return cudaErrorInvalidValue;
  return bf16 ? attn::launch<__nv_bfloat16>(a, layers, n_seq, s) : attn::launch<__half>(a, layers, n_seq, s);
}

}  // namespace net
}  // namespace fpb

// RefineNet / ScoreNet forward passes on the sm_100a kernels.
//
// Activation layout: planar buffers (include/fpk.h; 16-byte records of 8
// fp16/bf16 or 4 fp32 channels) on padded spatial grids, so every convolution
// is one fpk_gemm launch. FP16 / BF16 run kind::f16, FP32 and TF32 keep fp32
// activations and run kind::tf32 (TF32 multiplies, fp32 accumulation):
//   stem input   space-to-depth of the 160x160x6 crops, grid 83x83, 32 ch
//   stem 7x7/2   16 taps (4x4) over 32 ch              -> S2D, grid 41x41, 256 ch
//   conv 3x3/2   4 taps (2x2) over 256 ch              -> grid 41x41 (40x40 valid), 128 ch
//   res blocks   9 taps, shared zero row/column halo   (last one: CONCAT rendered|observed)
//   encAB        res blocks at 256 ch, last -> S2D grid 21x21, 1024 ch
//   conv 3x3/2   4 taps over 1024 ch                   -> grid 21x21 (20x20 valid), 512 ch
//   res blocks   last -> TOKENS [B*400, 512] + positional embedding
// Transformer layers run as GEMMs (QKV, out-proj, FF) + tcgen05 attention +
// LayerNorm + token mean; ScoreNet's cross-hypothesis attention is fp32.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "fp_net_kernels.cuh"
#include "fp_network.hpp"
#include "fp_profile.hpp"

namespace fpb {

namespace {

void check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
  }
}

constexpr int kStemGrid = 83;  // (160 + 7) / 2
constexpr int kG40 = 41;       // 40x40 valid + shared zero row/column
constexpr int kG20 = 21;
constexpr int kTokens = 400;
constexpr int kEmbed = 512;

}  // namespace

// ---------------------------------------------------------------------------
// Weight pack.
// ---------------------------------------------------------------------------

WeightPack WeightPack::load(const std::string& path) {
  std::ifstream in(path, std::ios::binary);
  if (!in) throw std::runtime_error("cannot open weight pack: " + path);
  std::vector<char> data((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
  if (data.size() < 16 || std::memcmp(data.data(), "FPW1", 4) != 0) {
    throw std::runtime_error("not a FoundationPose weight pack (.fpw): " + path);
  }
  uint32_t hdr[3];
  std::memcpy(hdr, data.data() + 4, 12);
  if (hdr[0] != 1) throw std::runtime_error("unsupported weight pack version in " + path);
  WeightPack p;
  p.arch = static_cast<int>(hdr[1]);
  const uint32_t count = hdr[2];
  if (16 + static_cast<size_t>(count) * 96 > data.size()) {
    throw std::runtime_error("truncated weight pack header: " + path);
  }
  for (uint32_t i = 0; i < count; ++i) {
    const char* rec = data.data() + 16 + 96 * i;
    char name[65] = {};
    std::memcpy(name, rec, 64);
    uint32_t ndim, shape[4];
    uint64_t offset;
    std::memcpy(&ndim, rec + 64, 4);
    std::memcpy(shape, rec + 68, 16);
    std::memcpy(&offset, rec + 88, 8);
    if (ndim > 4) throw std::runtime_error("bad tensor rank in " + path);
    size_t n = 1;
    std::vector<int> dims;
    for (uint32_t d = 0; d < ndim; ++d) {
      n *= shape[d];
      dims.push_back(static_cast<int>(shape[d]));
    }
    if (offset + n * 4 > data.size()) throw std::runtime_error("truncated tensor data in " + path);
    std::vector<float> v(n);
    std::memcpy(v.data(), data.data() + offset, n * 4);
    p.tensors[name] = std::move(v);
    p.shapes[name] = dims;
  }
  return p;
}

const std::vector<float>& WeightPack::at(const std::string& name) const {
  auto it = tensors.find(name);
  if (it == tensors.end()) throw std::runtime_error("weight pack is missing tensor " + name);
  return it->second;
}

// ---------------------------------------------------------------------------
// Weight arrangement.
// ---------------------------------------------------------------------------

namespace {

// [cout][taps][cin] -> chunk-major [cout][K'], k' = chunk*(taps*cw) + tap*cw + c,
// with cw = the channels of one 128-byte chunk (64 fp16/bf16, 32 fp32).
std::vector<float> chunkMajor(const std::vector<float>& w3, int cout, int taps, int cin, int chunk) {
  const int cw = cin < chunk ? cin : chunk;
  std::vector<float> out(static_cast<size_t>(cout) * taps * cin);
  for (int o = 0; o < cout; ++o)
    for (int t = 0; t < taps; ++t)
      for (int c = 0; c < cin; ++c) {
        const int chunk = c / cw;
        const size_t k = static_cast<size_t>(chunk) * taps * cw + static_cast<size_t>(t) * cw + (c % cw);
        out[static_cast<size_t>(o) * taps * cin + k] =
            w3[(static_cast<size_t>(o) * taps + t) * cin + c];
      }
  return out;
}

// fp32 -> TF32 (round to nearest, ties away from zero; the 13 low mantissa
// bits become zero) for weights consumed by kind::tf32 MMAs, which would
// otherwise truncate them.
std::vector<float> roundTf32(std::vector<float> v) {
  for (float& x : v) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) != 0x7F800000u) {  // finite
      u = (u + 0x1000u) & ~0x1FFFu;
      std::memcpy(&x, &u, 4);
    }
  }
  return v;
}

// Stride-1 kxk conv [cout][cin][k][k] -> [cout][k*k][cin].
std::vector<float> plainTaps(const std::vector<float>& w, int cout, int cin, int k) {
  std::vector<float> out(static_cast<size_t>(cout) * k * k * cin);
  for (int o = 0; o < cout; ++o)
    for (int c = 0; c < cin; ++c)
      for (int y = 0; y < k; ++y)
        for (int x = 0; x < k; ++x)
          out[(static_cast<size_t>(o) * k * k + y * k + x) * cin + c] =
              w[((static_cast<size_t>(o) * cin + c) * k + y) * k + x];
  return out;
}

// Stride-2 kxk conv over a space-to-depth input: taps (a, b) in nt x nt with
// nt = (k+1)/2, input channel (sub = dy*2+dx, c) at sub*cin_pad + c, kernel
// index (2a+dy, 2b+dx); taps past the kernel are zero. -> [cout][nt*nt][4*cin_pad].
std::vector<float> s2dTaps(const std::vector<float>& w, int cout, int cin, int k, int cin_pad) {
  const int nt = (k + 1) / 2;
  const int cs = 4 * cin_pad;
  std::vector<float> out(static_cast<size_t>(cout) * nt * nt * cs, 0.0f);
  for (int o = 0; o < cout; ++o)
    for (int a = 0; a < nt; ++a)
      for (int b = 0; b < nt; ++b)
        for (int dy = 0; dy < 2; ++dy)
          for (int dx = 0; dx < 2; ++dx) {
            const int ky = 2 * a + dy, kx = 2 * b + dx;
            if (ky >= k || kx >= k) continue;
            for (int c = 0; c < cin; ++c) {
              out[(static_cast<size_t>(o) * nt * nt + a * nt + b) * cs + (dy * 2 + dx) * cin_pad + c] =
                  w[((static_cast<size_t>(o) * cin + c) * k + ky) * k + kx];
            }
          }
  return out;
}

}  // namespace

class Network {
 public:
  // Uploads go through `setup`, a private non-blocking stream: no legacy-stream
  // work and no device-wide synchronisation, so a network can be built while
  // another thread captures a CUDA graph on the same device (group objects).
  Network(const WeightPack& pack, int dtype, std::vector<void*>& allocs, cudaStream_t setup)
      : dtype_(dtype), allocs_(allocs), arch_(pack.arch), setup_(setup) {
    // Encoder.
    conv("encA.conv1", pack, s2dTaps(pack.at("encA.conv1.w"), 64, 6, 7, 8), 64, 32, 16, offsets(4, kStemGrid),
         2.0 * 64 * 49 * 6);
    conv("encA.conv2", pack, s2dTaps(pack.at("encA.conv2.w"), 128, 64, 3, 64), 128, 256, 4, offsets(2, kG40),
         2.0 * 128 * 9 * 64);
    for (const char* r : {"encA.res1", "encA.res2"}) {
      plain3(std::string(r) + ".c1", pack, 128, kG40);
      plain3(std::string(r) + ".c2", pack, 128, kG40);
    }
    for (const char* r : {"encAB.res1", "encAB.res2"}) {
      plain3(std::string(r) + ".c1", pack, 256, kG40);
      plain3(std::string(r) + ".c2", pack, 256, kG40);
    }
    conv("encAB.conv", pack, s2dTaps(pack.at("encAB.conv.w"), 512, 256, 3, 256), 512, 1024, 4, offsets(2, kG20),
         2.0 * 512 * 9 * 256);
    for (const char* r : {"encAB.res3", "encAB.res4"}) {
      plain3(std::string(r) + ".c1", pack, 512, kG20);
      plain3(std::string(r) + ".c2", pack, 512, kG20);
    }
    pos = upload(pack.at("pos"));
    if (arch_ == 0) {
      // Both heads' QKV projections in one GEMM (3072 outputs).
      std::vector<float> w, b;
      for (const char* h : {"trans", "rot"}) {
        const auto& iw = pack.at(std::string(h) + ".attn.in_w");
        const auto& ib = pack.at(std::string(h) + ".attn.in_b");
        w.insert(w.end(), iw.begin(), iw.end());
        b.insert(b.end(), ib.begin(), ib.end());
      }
      layers["qkv"] = linear(w, b, 3 * 2 * kEmbed, kEmbed);
      for (const char* h : {"trans", "rot"}) {
        const std::string p(h);
        layers[p + ".out_proj"] = linear(pack.at(p + ".attn.out_w"), pack.at(p + ".attn.out_b"), kEmbed, kEmbed);
        layers[p + ".ff1"] = linear(pack.at(p + ".ff1.w"), pack.at(p + ".ff1.b"), kEmbed, kEmbed);
        layers[p + ".ff2"] = linear(pack.at(p + ".ff2.w"), pack.at(p + ".ff2.b"), kEmbed, kEmbed);
        f32[p + ".ln1.w"] = upload(pack.at(p + ".ln1.w"));
        f32[p + ".ln1.b"] = upload(pack.at(p + ".ln1.b"));
        f32[p + ".ln2.w"] = upload(pack.at(p + ".ln2.w"));
        f32[p + ".ln2.b"] = upload(pack.at(p + ".ln2.b"));
        f32[p + ".out.w"] = upload(pack.at(p + ".out.w"));
        f32[p + ".out.b"] = upload(pack.at(p + ".out.b"));
      }
    } else {
      layers["qkv"] = linear(pack.at("att.in_w"), pack.at("att.in_b"), 3 * kEmbed, kEmbed);
      layers["out_proj"] = linear(pack.at("att.out_w"), pack.at("att.out_b"), kEmbed, kEmbed);
      for (const char* n : {"att_cross.in_w", "att_cross.in_b", "att_cross.out_w", "att_cross.out_b",
                            "linear.w", "linear.b"}) {
        f32[n] = upload(pack.at(n));
      }
    }
    check(cudaStreamSynchronize(setup_), "weight upload");
  }

  const ConvLayer& L(const std::string& n) const {
    auto it = layers.find(n);
    if (it == layers.end()) throw std::runtime_error("network has no layer " + n);
    return it->second;
  }
  const float* F(const std::string& n) const { return f32.at(n); }

  std::map<std::string, ConvLayer> layers;
  std::map<std::string, float*> f32;
  float* pos = nullptr;
  int arch() const { return arch_; }

 private:
  static std::vector<int> offsets(int nt, int grid) {
    std::vector<int> o;
    for (int a = 0; a < nt; ++a)
      for (int b = 0; b < nt; ++b) o.push_back(a * grid + b);
    return o;
  }

  float* upload(const std::vector<float>& v) {
    void* p = nullptr;
    check(cudaMalloc(&p, v.size() * 4 + 16), "cudaMalloc weights");
    allocs_.push_back(p);
    // From pageable memory the call returns once `v` has been staged.
    check(cudaMemcpyAsync(p, v.data(), v.size() * 4, cudaMemcpyHostToDevice, setup_), "upload weights");
    return static_cast<float*>(p);
  }

  // Strict FP32: the part of each weight below its TF32 rounding, itself
  // rounded to TF32 (the hi * W_lo product of the three-term split).
  void* uploadWeightRemainder(const std::vector<float>& v) {
    const std::vector<float> hi = roundTf32(v);
    std::vector<float> lo(v.size());
    for (size_t i = 0; i < v.size(); ++i) lo[i] = v[i] - hi[i];
    return upload(roundTf32(lo));
  }

  // Weights in the activation type: fp32 as is, else converted on the device.
  void* uploadWeights(const std::vector<float>& v) {
    if (dtype_ == FPK_DTYPE_F32 || dtype_ == FPK_DTYPE_F32_EXACT) return upload(roundTf32(v));
    float* tmp = nullptr;
    check(cudaMallocAsync(reinterpret_cast<void**>(&tmp), v.size() * 4, setup_), "cudaMallocAsync staging");
    check(cudaMemcpyAsync(tmp, v.data(), v.size() * 4, cudaMemcpyHostToDevice, setup_), "upload staging");
    void* p = nullptr;
    check(cudaMalloc(&p, v.size() * 2 + 16), "cudaMalloc weights");
    allocs_.push_back(p);
    check(net::launchConvert(tmp, p, static_cast<long long>(v.size()), dtype_ == FPK_DTYPE_BF16, setup_),
          "convert weights");
    check(cudaFreeAsync(tmp, setup_), "cudaFreeAsync staging");
    return p;
  }

  void conv(const std::string& name, const WeightPack& pack, const std::vector<float>& taps_w,
            int cout, int cin, int taps, const std::vector<int>& offs, double flops_per_row) {
    ConvLayer c;
    c.flops_per_row = flops_per_row;
    const std::vector<float> cm = chunkMajor(taps_w, cout, taps, cin, chunk());
    c.w = uploadWeights(cm);
    if (dtype_ == FPK_DTYPE_F32_EXACT) c.w_lo = uploadWeightRemainder(cm);
    c.bias = upload(pack.at(name + ".b"));
    c.cin = cin;
    c.cout = cout;
    c.taps = taps;
    for (int t = 0; t < taps; ++t) c.tap_off[t] = offs[t];
    layers[name] = c;
  }

  void plain3(const std::string& name, const WeightPack& pack, int ch, int grid) {
    std::vector<int> offs;
    for (int ky = 0; ky < 3; ++ky)
      for (int kx = 0; kx < 3; ++kx) offs.push_back((ky - 1) * grid + (kx - 1));
    conv(name, pack, plainTaps(pack.at(name + ".w"), ch, ch, 3), ch, ch, 9, offs, 2.0 * ch * 9 * ch);
  }

  ConvLayer linear(const std::vector<float>& w, const std::vector<float>& b, int cout, int cin) {
    ConvLayer c;
    const std::vector<float> cm = chunkMajor(w, cout, 1, cin, chunk());
    c.w = uploadWeights(cm);
    if (dtype_ == FPK_DTYPE_F32_EXACT) c.w_lo = uploadWeightRemainder(cm);
    c.bias = upload(b);
    c.cin = cin;
    c.cout = cout;
    c.taps = 1;
    c.flops_per_row = 2.0 * cout * cin;
    return c;
  }

  int chunk() const { return (dtype_ == FPK_DTYPE_F32 || dtype_ == FPK_DTYPE_F32_EXACT) ? 32 : 64; }

  int dtype_;
  std::vector<void*>& allocs_;
  int arch_;
  cudaStream_t setup_;
};

// ---------------------------------------------------------------------------
// Activation workspace.
// ---------------------------------------------------------------------------

struct NetworkRunner::Act {
  Planar x1, e[3], ab[3], x4, f[3], tok, qkv, att, y1, x1n, h, y2;
  float* feat = nullptr;     // [2][B][512]
  float* qkvc = nullptr;     // [B][1536]
  float* oc = nullptr;       // [B][512]
  float* xc = nullptr;       // [B][512]
};

namespace {

// Planar buffer of `channels` channels, `per_record` channels per 16-byte
// record (8 for fp16/bf16, 4 for fp32).
Planar allocPlanar(std::vector<void*>& allocs, long long rows, int channels, int per_record, cudaStream_t setup) {
  Planar p;
  p.rows = rows;
  p.planes = channels / per_record;
  p.plane_stride = ((kGuardPre + rows + kGuardPost) * 16 + 255) / 256 * 256;
  p.bytes = static_cast<size_t>(p.plane_stride) * p.planes;
  check(cudaMalloc(&p.mem, p.bytes), "cudaMalloc activations");
  allocs.push_back(p.mem);
  check(cudaMemsetAsync(p.mem, 0, p.bytes, setup), "zero activations");
  p.base = static_cast<unsigned char*>(p.mem) + kGuardPre * 16;
  return p;
}

float* allocF32(std::vector<void*>& allocs, size_t n) {
  void* p = nullptr;
  check(cudaMalloc(&p, n * 4), "cudaMalloc");
  allocs.push_back(p);
  return static_cast<float*>(p);
}

}  // namespace

NetworkRunner::NetworkRunner(const std::string& refine_path, const std::string& score_path,
                             NetPrecision precision, int max_batch, int crop_w, int crop_h)
    : precision_(precision), max_batch_(max_batch), crop_w_(crop_w), crop_h_(crop_h) {
  if (crop_w != 160 || crop_h != 160) {
    throw std::runtime_error("the built-in RefineNet/ScoreNet require 160x160 crops");
  }
  if (max_batch <= 0 || max_batch > 1024) throw std::runtime_error("max batch must be in [1, 1024]");
  const int dt = dtype();
  const int pr = perRecord();
  cudaStream_t setup = nullptr;
  check(cudaStreamCreateWithFlags(&setup, cudaStreamNonBlocking), "set-up stream");
  try {
    WeightPack rp = WeightPack::load(refine_path);
    WeightPack sp = WeightPack::load(score_path);
    if (rp.arch != 0) throw std::runtime_error(refine_path + " is not a RefineNet pack");
    if (sp.arch != 1) throw std::runtime_error(score_path + " is not a ScoreNet pack");
    refine_ = std::make_unique<Network>(rp, dt, allocations_, setup);
    score_ = std::make_unique<Network>(sp, dt, allocations_, setup);
    const long long B = max_batch;
    const long long N = 2 * B;
    stem_ = allocPlanar(allocations_, N * kStemGrid * kStemGrid, 32, pr, setup);
    act_ = std::make_unique<Act>();
    Act& a = *act_;
    a.x1 = allocPlanar(allocations_, N * kG40 * kG40, 256, pr, setup);
    for (auto& p : a.e) p = allocPlanar(allocations_, N * kG40 * kG40, 128, pr, setup);
    for (auto& p : a.ab) p = allocPlanar(allocations_, B * kG40 * kG40, 256, pr, setup);
    a.x4 = allocPlanar(allocations_, B * kG20 * kG20, 1024, pr, setup);
    for (auto& p : a.f) p = allocPlanar(allocations_, B * kG20 * kG20, 512, pr, setup);
    const long long T = B * kTokens;
    a.tok = allocPlanar(allocations_, T, kEmbed, pr, setup);
    a.qkv = allocPlanar(allocations_, T, 6 * kEmbed, pr, setup);
    a.att = allocPlanar(allocations_, T, 2 * kEmbed, pr, setup);
    a.y1 = allocPlanar(allocations_, T, kEmbed, pr, setup);
    a.x1n = allocPlanar(allocations_, T, kEmbed, pr, setup);
    a.h = allocPlanar(allocations_, T, kEmbed, pr, setup);
    a.y2 = allocPlanar(allocations_, T, kEmbed, pr, setup);
    a.feat = allocF32(allocations_, 2 * B * kEmbed);
    a.qkvc = allocF32(allocations_, B * 3 * kEmbed);
    a.oc = allocF32(allocations_, B * kEmbed);
    a.xc = allocF32(allocations_, B * kEmbed);
    void* e = nullptr;
    check(cudaMalloc(&e, 16), "cudaMalloc error flag");
    allocations_.push_back(e);
    check(cudaMemsetAsync(e, 0, 16, setup), "zero error flag");
    err_ = static_cast<int*>(e);
    if (dt == FPK_DTYPE_F32_EXACT) {
      // Largest split activation (a GEMM input: x1, 2B images x 41^2 rows x
      // 256 channels) and partial sum (a GEMM output on its input's grid: the
      // RefineNet QKV output, B x 400 rows x 3072 channels, or the stem's 64
      // channels on the 83^2 grid).
      auto planar_bytes = [](long long rows, int channels) {
        return static_cast<size_t>(((kGuardPre + rows + kGuardPost) * 16 + 255) / 256 * 256) * (channels / 4);
      };
      split_bytes_ = std::max(planar_bytes(N * kG40 * kG40, 256), planar_bytes(N * kStemGrid * kStemGrid, 32));
      split_bytes_ = std::max(split_bytes_, planar_bytes(B * kG20 * kG20, 1024));
      partial_bytes_ = std::max(planar_bytes(N * kStemGrid * kStemGrid, 64), planar_bytes(B * kTokens, 6 * kEmbed));
      for (void** p : {&split_hi_, &split_lo_, &partial_[0], &partial_[1]}) {
        const size_t bytes = (p == &split_hi_ || p == &split_lo_) ? split_bytes_ : partial_bytes_;
        check(cudaMalloc(p, bytes), "cudaMalloc strict-FP32 scratch");
        allocations_.push_back(*p);
      }
    }
    splitk_bytes_ = 24ll << 20;
    check(cudaMalloc(&splitk_, static_cast<size_t>(splitk_bytes_)), "cudaMalloc split-K scratch");
    allocations_.push_back(splitk_);
    check(cudaStreamSynchronize(setup), "network set-up");
    cudaStreamDestroy(setup);
  } catch (...) {
    cudaStreamSynchronize(setup);
    cudaStreamDestroy(setup);
    for (void* p : allocations_) cudaFree(p);
    allocations_.clear();
    throw;
  }
}

void NetworkRunner::clearError(cudaStream_t s) { check(cudaMemsetAsync(err_, 0, sizeof(int), s), "reset error flag"); }

NetworkRunner::~NetworkRunner() {
  for (void* p : allocations_) cudaFree(p);
}

int NetworkRunner::dtype() const {
  switch (precision_) {
    case NetPrecision::kBF16:
      return FPK_DTYPE_BF16;
    case NetPrecision::kFP16:
      return FPK_DTYPE_F16;
    case NetPrecision::kTF32:
      return FPK_DTYPE_F32;  // fp32 activations rounded to TF32, TF32 tensor-core products
    default:
      return FPK_DTYPE_F32_EXACT;  // FP32: fp32 activations, split-operand products (fp32-accurate)
  }
}

int NetworkRunner::perRecord() const {
  return (dtype() == FPK_DTYPE_F32 || dtype() == FPK_DTYPE_F32_EXACT) ? 4 : 8;
}

void NetworkRunner::gemm(const ConvLayer& L, const Planar& a, long long a_row0, long long rows,
                         const Planar& dst, int mode, int img_rows, int grid_w, int valid_h,
                         int valid_w, bool relu, const Planar* residual, int dst_img_rows,
                         int dst_grid_w, int img_mod, int ch_step, const float* pos,
                         cudaStream_t s, long long dst_row0, int a_plane0) {
  fpk_gemm_desc_t d{};
  d.a = a.base + a_row0 * 16 + static_cast<long long>(a_plane0) * a.plane_stride;
  d.a_plane_stride = a.plane_stride;
  d.rows = static_cast<int>(rows);
  d.cin = L.cin;
  d.taps = L.taps;
  for (int t = 0; t < L.taps; ++t) d.tap_off[t] = L.tap_off[t];
  d.w = L.w;
  d.cout = L.cout;
  d.bias = L.bias;
  d.residual = residual != nullptr ? residual->base : nullptr;
  d.res_plane_stride = residual != nullptr ? residual->plane_stride : 0;
  d.relu = relu ? 1 : 0;
  d.dst = dst.base + dst_row0 * 16;
  d.dst_plane_stride = dst.plane_stride;
  d.dst_mode = mode;
  d.img_rows = img_rows;
  d.grid_w = grid_w;
  d.valid_h = valid_h;
  d.valid_w = valid_w;
  d.dst_img_rows = dst_img_rows;
  d.dst_grid_w = dst_grid_w;
  d.img_mod = img_mod;
  d.ch_step = ch_step;
  d.pos = pos;
  d.dtype = dtype();
  d.error_flag = err_;
  d.splitk_ws = split_k_ ? splitk_ : nullptr;
  d.splitk_ws_bytes = split_k_ ? splitk_bytes_ : 0;
  const double valid_rows = static_cast<double>(rows / img_rows) * valid_h * valid_w;
  prof::Scope scope(prof::kGemm, valid_rows * L.flops_per_row, s);
  if (d.dtype == FPK_DTYPE_F32_EXACT) {
    exactGemm(d, L, s);
    return;
  }
  if (fpk_gemm(&d, s) != 0) throw std::runtime_error(fpk_last_error());
}

// Strict FP32 layer: A is split into TF32 hi and lo parts, and the layer is
//   P1  = A_hi W_hi + bias + residual        (SAME layout on A's grid)
//   P2  = A_hi W_lo + P1
//   out = A_lo W_hi + P2, then ReLU / destination layout / embedding,
// every partial kept in fp32. The dropped A_lo W_lo term is below 2^-20 of
// the product, so the result carries fp32 accuracy (the reference's FP32
// engines run fp32 arithmetic, src/tensorrt_runner.cu:65-80).
void NetworkRunner::exactGemm(const fpk_gemm_desc_t& d, const ConvLayer& L, cudaStream_t s) {
  auto stride_for = [](long long rows) { return ((kGuardPre + rows + kGuardPost) * 16 + 255) / 256 * 256; };
  const int a_planes = d.cin / 4;
  const long long a_stride = stride_for(d.rows);
  const long long p_stride = stride_for(d.rows);
  if (static_cast<size_t>(a_stride) * a_planes > split_bytes_ ||
      static_cast<size_t>(p_stride) * (d.cout / 4) > partial_bytes_) {
    throw std::runtime_error("strict-FP32 scratch too small for a layer");
  }
  unsigned char* hi = static_cast<unsigned char*>(split_hi_) + kGuardPre * 16;
  unsigned char* lo = static_cast<unsigned char*>(split_lo_) + kGuardPre * 16;
  check(net::launchSplitTf32(static_cast<const unsigned char*>(d.a), d.a_plane_stride, hi, lo, a_stride, d.rows,
                             a_planes, static_cast<int>(kGuardPre), static_cast<int>(kGuardPost), s),
        "split operands");
  unsigned char* p1 = static_cast<unsigned char*>(partial_[0]) + kGuardPre * 16;
  unsigned char* p2 = static_cast<unsigned char*>(partial_[1]) + kGuardPre * 16;
  fpk_gemm_desc_t g = d;
  // P1: A_hi W_hi + bias + residual.
  g.a = hi;
  g.a_plane_stride = a_stride;
  g.w = L.w;
  g.relu = 0;
  g.dst = p1;
  g.dst_plane_stride = p_stride;
  g.dst_mode = FPK_DST_SAME;
  g.pos = nullptr;
  if (fpk_gemm(&g, s) != 0) throw std::runtime_error(fpk_last_error());
  // P2: A_hi W_lo + P1.
  g.w = L.w_lo;
  g.bias = nullptr;
  g.residual = p1;
  g.res_plane_stride = p_stride;
  g.dst = p2;
  if (fpk_gemm(&g, s) != 0) throw std::runtime_error(fpk_last_error());
  // out: A_lo W_hi + P2 through the layer's own epilogue.
  g = d;
  g.a = lo;
  g.a_plane_stride = a_stride;
  g.w = L.w;
  g.bias = nullptr;
  g.residual = p2;
  g.res_plane_stride = p_stride;
  if (fpk_gemm(&g, s) != 0) throw std::runtime_error(fpk_last_error());
}

// Encoder for n hypotheses whose 2n images start at stem row `stem_row0`;
// leaves the tokens (+ positional embedding) in act_->tok rows [0, n*400).
void NetworkRunner::encoder(const Network& net, int n, long long stem_row0, cudaStream_t s) {
  Act& a = *act_;
  const int N = 2 * n;
  const int i40 = kG40 * kG40;
  const int i20 = kG20 * kG20;
  // encoder A (both crops, shared weights)
  gemm(net.L("encA.conv1"), stem_, stem_row0, static_cast<long long>(N) * kStemGrid * kStemGrid, a.x1,
       FPK_DST_S2D, kStemGrid * kStemGrid, kStemGrid, 80, 80, true, nullptr, i40, kG40, 1, 0, nullptr, s);
  const long long r40 = static_cast<long long>(N) * i40;
  gemm(net.L("encA.conv2"), a.x1, 0, r40, a.e[0], FPK_DST_SAME, i40, kG40, 40, 40, true, nullptr, 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encA.res1.c1"), a.e[0], 0, r40, a.e[1], FPK_DST_SAME, i40, kG40, 40, 40, true, nullptr, 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encA.res1.c2"), a.e[1], 0, r40, a.e[2], FPK_DST_SAME, i40, kG40, 40, 40, true, &a.e[0], 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encA.res2.c1"), a.e[2], 0, r40, a.e[0], FPK_DST_SAME, i40, kG40, 40, 40, true, nullptr, 0, 0, 1, 0, nullptr, s);
  // Last block writes rendered images to channels 0..127 and observed to 128..255.
  gemm(net.L("encA.res2.c2"), a.e[0], 0, r40, a.ab[0], FPK_DST_CONCAT, i40, kG40, 40, 40, true, &a.e[2], 0, 0, n, 128, nullptr, s);
  // encoder AB
  const long long rab = static_cast<long long>(n) * i40;
  gemm(net.L("encAB.res1.c1"), a.ab[0], 0, rab, a.ab[1], FPK_DST_SAME, i40, kG40, 40, 40, true, nullptr, 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encAB.res1.c2"), a.ab[1], 0, rab, a.ab[2], FPK_DST_SAME, i40, kG40, 40, 40, true, &a.ab[0], 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encAB.res2.c1"), a.ab[2], 0, rab, a.ab[0], FPK_DST_SAME, i40, kG40, 40, 40, true, nullptr, 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encAB.res2.c2"), a.ab[0], 0, rab, a.x4, FPK_DST_S2D, i40, kG40, 40, 40, true, &a.ab[2], i20, kG20, 1, 0, nullptr, s);
  const long long r20 = static_cast<long long>(n) * i20;
  gemm(net.L("encAB.conv"), a.x4, 0, r20, a.f[0], FPK_DST_SAME, i20, kG20, 20, 20, true, nullptr, 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encAB.res3.c1"), a.f[0], 0, r20, a.f[1], FPK_DST_SAME, i20, kG20, 20, 20, true, nullptr, 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encAB.res3.c2"), a.f[1], 0, r20, a.f[2], FPK_DST_SAME, i20, kG20, 20, 20, true, &a.f[0], 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encAB.res4.c1"), a.f[2], 0, r20, a.f[0], FPK_DST_SAME, i20, kG20, 20, 20, true, nullptr, 0, 0, 1, 0, nullptr, s);
  gemm(net.L("encAB.res4.c2"), a.f[0], 0, r20, a.tok, FPK_DST_TOKENS, i20, kG20, 20, 20, true, &a.f[2], 0, 0, 1, 0, net.pos, s);
}

void NetworkRunner::refine(int count, int first_chunk, float* delta_t, float* delta_r, cudaStream_t s) {
  if (count <= 0 || count > max_batch_) throw std::runtime_error("refine batch exceeds the prepared maximum");
  split_k_ = count == 1;
  Act& a = *act_;
  const Network& net = *refine_;
  const int dt = dtype();
  const int pr = perRecord();
  encoder(net, count, static_cast<long long>(first_chunk) * 2 * count * kStemGrid * kStemGrid, s);
  const long long T = static_cast<long long>(count) * kTokens;
  const int t = static_cast<int>(T);
  gemm(net.L("qkv"), a.tok, 0, T, a.qkv, FPK_DST_SAME, t, 1, t, 1, false, nullptr, 0, 0, 1, 0, nullptr, s);
  net::AttnArgs at{};
  at.qkv = a.qkv.base;
  at.qkv_plane_stride = a.qkv.plane_stride;
  at.qkv_layer_planes = 3 * kEmbed / pr;
  at.q_plane = 0;
  at.k_plane = kEmbed / pr;
  at.v_plane = 2 * kEmbed / pr;
  at.out = a.att.base;
  at.out_plane_stride = a.att.plane_stride;
  at.out_layer_planes = kEmbed / pr;
  at.seq_len = kTokens;
  at.heads = 4;
  at.scale_log2 = 1.4426950408889634f / std::sqrt(128.0f);
  at.error_flag = err_;
  {
    prof::Scope scope(prof::kAttention, 2.0 * 4 * count * 4.0 * kTokens * kTokens * 128, s);
    check(net::launchAttentionTc(at, 2, count, dt, s), "attention");
  }
  float* outs[2] = {delta_t, delta_r};
  const char* heads[2] = {"trans", "rot"};
  for (int z = 0; z < 2; ++z) {
    const std::string p(heads[z]);
    // y1 = x + out_proj(attention); x1 = LN1(y1); y2 = x1 + FF(x1); z = LN2(y2)
    gemm(net.L(p + ".out_proj"), a.att, 0, T, a.y1, FPK_DST_SAME, t, 1, t, 1, false, &a.tok, 0, 0, 1, 0, nullptr, s, 0, z * kEmbed / pr);
    net::LnArgs ln{a.y1.base, a.y1.plane_stride, a.x1n.base, a.x1n.plane_stride, T, net.F(p + ".ln1.w"), net.F(p + ".ln1.b"), 1e-5f};
    check(net::launchLayerNorm(ln, dt, s), "layernorm");
    gemm(net.L(p + ".ff1"), a.x1n, 0, T, a.h, FPK_DST_SAME, t, 1, t, 1, true, nullptr, 0, 0, 1, 0, nullptr, s);
    gemm(net.L(p + ".ff2"), a.h, 0, T, a.y2, FPK_DST_SAME, t, 1, t, 1, false, &a.x1n, 0, 0, 1, 0, nullptr, s);
    net::LnArgs ln2{a.y2.base, a.y2.plane_stride, a.y1.base, a.y1.plane_stride, T, net.F(p + ".ln2.w"), net.F(p + ".ln2.b"), 1e-5f};
    check(net::launchLayerNorm(ln2, dt, s), "layernorm");
    float* feat = a.feat + static_cast<size_t>(z) * max_batch_ * kEmbed;
    check(net::launchTokenMean(a.y1.base, a.y1.plane_stride, kTokens, count, feat, dt, s), "token mean");
    check(net::launchLinearF32(feat, net.F(p + ".out.w"), net.F(p + ".out.b"), outs[z], count, 3, kEmbed, false, s), "head");
  }
}

void NetworkRunner::score(int n, float* scores, cudaStream_t s) {
  scoreFeatures(n, act_->feat, s);
  scoreHead(n, act_->feat, scores, s);
}

void NetworkRunner::scoreFeatures(int n, float* features, cudaStream_t s) {
  if (n <= 0 || n > max_batch_) throw std::runtime_error("score batch exceeds the prepared maximum");
  split_k_ = n == 1;
  Act& a = *act_;
  const Network& net = *score_;
  const int dt = dtype();
  const int pr = perRecord();
  encoder(net, n, 0, s);
  const long long T = static_cast<long long>(n) * kTokens;
  const int t = static_cast<int>(T);
  gemm(net.L("qkv"), a.tok, 0, T, a.qkv, FPK_DST_SAME, t, 1, t, 1, false, nullptr, 0, 0, 1, 0, nullptr, s);
  net::AttnArgs at{};
  at.qkv = a.qkv.base;
  at.qkv_plane_stride = a.qkv.plane_stride;
  at.qkv_layer_planes = 3 * kEmbed / pr;
  at.q_plane = 0;
  at.k_plane = kEmbed / pr;
  at.v_plane = 2 * kEmbed / pr;
  at.out = a.att.base;
  at.out_plane_stride = a.att.plane_stride;
  at.out_layer_planes = kEmbed / pr;
  at.seq_len = kTokens;
  at.heads = 4;
  at.scale_log2 = 1.4426950408889634f / std::sqrt(128.0f);
  at.error_flag = err_;
  {
    prof::Scope scope(prof::kAttention, 1.0 * 4 * n * 4.0 * kTokens * kTokens * 128, s);
    check(net::launchAttentionTc(at, 1, n, dt, s), "attention");
  }
  gemm(net.L("out_proj"), a.att, 0, T, a.y1, FPK_DST_SAME, t, 1, t, 1, false, nullptr, 0, 0, 1, 0, nullptr, s);
  check(net::launchTokenMean(a.y1.base, a.y1.plane_stride, kTokens, n, features, dt, s), "token mean");
}

void NetworkRunner::scoreHead(int n, const float* features, float* scores, cudaStream_t s) {
  if (n <= 0 || n > max_batch_) throw std::runtime_error("score batch exceeds the prepared maximum");
  Act& a = *act_;
  const Network& net = *score_;
  // Attention across the n hypotheses (fp32), then the score head.
  check(net::launchLinearF32(features, net.F("att_cross.in_w"), net.F("att_cross.in_b"), a.qkvc, n, 3 * kEmbed, kEmbed, false, s), "cross qkv");
  check(net::launchSmallAttention(a.qkvc, n, a.oc, s), "cross attention");
  check(net::launchLinearF32(a.oc, net.F("att_cross.out_w"), net.F("att_cross.out_b"), a.xc, n, kEmbed, kEmbed, false, s), "cross out");
  check(net::launchLinearF32(a.xc, net.F("linear.w"), net.F("linear.b"), scores, n, 1, kEmbed, false, s), "score head");
}

void NetworkRunner::loadNchw(const float* rendered, const float* observed, int n, cudaStream_t s) {
  if (n <= 0 || n > max_batch_) throw std::runtime_error("batch exceeds the prepared maximum");
  check(net::launchNchwToStem(rendered, observed, n, crop_h_, crop_w_, stem_.base, stem_.plane_stride,
                              dtype(), s),
        "nchw to stem");
}

namespace {
double convFlops(double cout, double cin, double k, double hw) { return 2.0 * cout * cin * k * k * hw; }

double encoderFlopsPerHyp() {
  double f = 2 * convFlops(64, 6, 7, 6400) + 2 * convFlops(128, 64, 3, 1600);
  f += 2 * 4 * convFlops(128, 128, 3, 1600);
  f += 4 * convFlops(256, 256, 3, 1600) + convFlops(512, 256, 3, 400) + 4 * convFlops(512, 512, 3, 400);
  return f;
}

double mhaFlops(double L, double E) {
  return 2.0 * L * E * 3 * E + 4.0 * L * L * E + 2.0 * L * E * E;
}
}  // namespace

double NetworkRunner::refineFlopsPerHyp() const {
  const double layer = mhaFlops(kTokens, kEmbed) + 2 * 2.0 * kTokens * kEmbed * kEmbed;
  return encoderFlopsPerHyp() + 2 * layer;
}

double NetworkRunner::scoreFlopsPerHyp() const {
  return encoderFlopsPerHyp() + mhaFlops(kTokens, kEmbed);
}

}  // namespace fpb

// ---------------------------------------------------------------------------
// C ABI.
// ---------------------------------------------------------------------------

struct fpk_net {
  std::unique_ptr<fpb::NetworkRunner> runner;
};

namespace fpb {
int fail(const std::string& msg);
}

extern "C" {

fpk_net_t* fpk_net_create(const char* refine_pack, const char* score_pack, int precision, int max_batch) {
  try {
    if (refine_pack == nullptr || score_pack == nullptr) {
      fpb::fail("fpk_net_create: weight pack paths are required");
      return nullptr;
    }
    auto n = std::make_unique<fpk_net>();
    n->runner = std::make_unique<fpb::NetworkRunner>(refine_pack, score_pack,
                                                     static_cast<fpb::NetPrecision>(precision), max_batch,
                                                     160, 160);
    return n.release();
  } catch (const std::exception& e) {
    fpb::fail(e.what());
    return nullptr;
  }
}

void fpk_net_destroy(fpk_net_t* net) { delete net; }

int fpk_net_refine(fpk_net_t* net, const float* rendered, const float* observed, int n, float* trans,
                   float* rot, void* stream) {
  try {
    if (net == nullptr) return fpb::fail("fpk_net_refine: null handle");
    auto s = static_cast<cudaStream_t>(stream);
    net->runner->loadNchw(rendered, observed, n, s);
    net->runner->refine(n, 0, trans, rot, s);
    return 0;
  } catch (const std::exception& e) {
    return fpb::fail(e.what());
  }
}

int fpk_net_score(fpk_net_t* net, const float* rendered, const float* observed, int n, float* scores,
                  void* stream) {
  try {
    if (net == nullptr) return fpb::fail("fpk_net_score: null handle");
    auto s = static_cast<cudaStream_t>(stream);
    net->runner->loadNchw(rendered, observed, n, s);
    net->runner->score(n, scores, s);
    return 0;
  } catch (const std::exception& e) {
    return fpb::fail(e.what());
  }
}

int fpk_net_error(fpk_net_t* net, int* host_flag) {
  if (net == nullptr || host_flag == nullptr) return fpb::fail("fpk_net_error: null argument");
  const cudaError_t e = cudaMemcpy(host_flag, net->runner->errorFlag(), sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fpb::fail(cudaGetErrorString(e));
  return 0;
}

}  // extern "C"

// SpectroStream decode phase: weights in implicit-GEMM layouts, the launch
// plan of one decode (dequantise -> decoder -> output conv -> iSTFT), its
// CUDA graph, and the C ABI of include/mrtss.h.
//
// Reference (rhymeswithlion/magenta-realtime-mlx-cpp):
//   codec block of System::generate_chunk  system.cpp:372-390
//   SpectroStreamDecoder                   spectrostream.cpp:340-419
//   istft_postprocess                      spectrostream.cpp:593-681
//   rvq_dequantization                     rvq.cpp:68-87
#include <cuda_runtime.h>

#include <array>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/mrtss.h"
#include "codec_kernels.cuh"
#include "device_errors.h"
#include "host_util.h"

using namespace mrtdf;

namespace {

#define SS_CUDA(expr)                                                                                    \
  do {                                                                                                   \
    cudaError_t e_ = (expr);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      throw Error{MRTDF_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)};                   \
  } while (0)


// Decoder block table (dec_block_specs, spectrostream.cpp:328-338): in, out,
// stride (h, w), transposed kernel (h, w); every post kernel is 3 x 3.
struct DecSpec {
  int in, out, sh, sw, tkh, tkw;
};
constexpr DecSpec kDec[7] = {{512, 1024, 2, 1, 4, 3}, {512, 256, 2, 2, 4, 4}, {256, 256, 1, 2, 3, 4},
                             {256, 256, 1, 2, 3, 4},  {256, 128, 1, 3, 3, 6}, {128, 128, 1, 2, 3, 4},
                             {128, 64, 1, 2, 3, 4}};
constexpr int kEmb = 256, kProj = 2560, kUnfold = 5, kCrop = 4, kFft = 960, kHop = 480, kOutCh = 64;
constexpr int kCodebookSize = 1024;  // codec_rvq_codebook_size (system.h:51)

int floor_div(int a, int b) { return a >= 0 ? a / b : -((-a + b - 1) / b); }
int ceil_div(int a, int b) { return -floor_div(-a, b); }

// Tensors of the decoder bundle in construction order, canonical layouts.
struct CodecSpec {
  std::string key;
  std::vector<int64_t> shape;
  float stddev;
};

std::vector<CodecSpec> codec_specs() {
  std::vector<CodecSpec> v;
  auto conv = [&](const std::string& p, int O, int I, int kh, int kw) {
    v.push_back({p + ".weight", {O, I, kh, kw}, 1.0f / std::sqrt((float)I * kh * kw)});
    v.push_back({p + ".bias", {O}, 0.02f});
  };
  conv("input_proj.conv1", kProj, kEmb, 1, 1);
  conv("input_proj.conv2", kProj, kProj, 1, 1);
  conv("input_proj.shortcut", kProj, kEmb, 1, 1);
  conv("input_conv.conv1", 512, 512, 3, 3);
  conv("input_conv.conv2", 512, 512, 3, 3);
  for (int i = 0; i < 7; ++i) {
    const DecSpec& s = kDec[i];
    const std::string p = "decoder_blocks." + std::to_string(i);
    // transposed conv (I, O, kh, kw): each output sees ~I kh kw / (sh sw) inputs
    v.push_back({p + ".conv_transpose.weight", {s.in, s.out, s.tkh, s.tkw},
                 1.0f / std::sqrt((float)s.in * s.tkh * s.tkw / (s.sh * s.sw))});
    v.push_back({p + ".conv_transpose.bias", {s.out}, 0.02f});
    conv(p + ".conv", s.out, s.out, 3, 3);
    if (s.in != s.out) conv(p + ".shortcut", s.out, s.in, 1, 1);
  }
  conv("output_conv", 2, kOutCh, 7, 7);
  return v;
}

struct DevConv {
  float* w = nullptr;  // (cout, ntaps, cin)
  float* b = nullptr;  // (cout)
  int cout = 0, cin = 0, ntaps = 1, ntx = 1;
};

struct Host4 {
  const float* p;
  int n, h, w, c;
};

}  // namespace

struct mrtss_codec {
  int device = 0, max_batch = 1, max_frames = 1;
  bool loaded = false;
  cudaStream_t s = nullptr;
  std::vector<void*> allocs;
  void* weights = nullptr;
  DevConv ip_c1, ip_c2, ip_sc, ic_c1, ic_c2;
  DevConv ct[7][6];
  int nphase[7] = {};
  int phase_ry[7][6] = {}, phase_rx[7][6] = {};
  DevConv post[7], sc[7];
  bool has_sc[7] = {};
  float* oc_w = nullptr;
  float* oc_b = nullptr;
  float* codebooks = nullptr;
  int K = 0, C = 0, D = 0;
  float* synth = nullptr;
  float* cosv = nullptr;
  // activations and I/O (float32 unless noted)
  float* x0 = nullptr;  // (B, S + 1, 1, 256)
  float* raw[2] = {nullptr, nullptr};
  float* elu = nullptr;
  float* y = nullptr;
  float* r = nullptr;
  float* spec = nullptr;   // (B, 4 S, 480, 4)
  float* audio = nullptr;  // (B, S * 1920, 2)
  int32_t* codes = nullptr;
  int* err = nullptr;
  size_t act_floats = 0, x0_floats = 0, spec_floats = 0, audio_floats = 0, codes_ints = 0;
  std::map<std::array<int, 3>, cudaGraphExec_t> graphs;
  ~mrtss_codec() {
    if (device >= 0) cudaSetDevice(device);
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    if (weights) cudaFree(weights);
    for (void* p : allocs) cudaFree(p);
    if (s) cudaStreamDestroy(s);
  }
};

namespace {

// ---- launch plan ---------------------------------------------------------------
// Walks one decode at (B, S). With launch = false it only counts kernels and
// the largest activation each buffer must hold; with launch = true it
// enqueues every kernel on the codec's stream.
struct Plan {
  mrtss_codec* c;
  bool launch;
  bool pdl = true;
  long long kernels = 0;
  size_t need_act = 0;
  int nseq = 1;  // sequences in the call: the split-K choice uses one sequence's tiles

  void fail(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw Error{MRTDF_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e)};
  }
  void run(const ConvParams& p) {
    ++kernels;
    need_act = std::max(need_act, (size_t)p.in_n * p.in_h * p.in_w * p.cin);
    const size_t out_px = (size_t)(p.split > 0 ? p.n_img * (p.cout / p.split) : p.n_img) * p.ho * p.wo;
    need_act = std::max(need_act, out_px * (size_t)(p.split > 0 ? p.split : p.cout));
    if (launch) fail(launch_conv_tc(p, c->err, c->s, pdl), "conv_tc");
  }

  static void tile(ConvParams& p) {
    p.wt = std::min(p.wq, 128);
    p.ht = std::max(1, std::min(p.hq, 128 / p.wt));
    p.tiles_x = (p.wq + p.wt - 1) / p.wt;
    p.tiles_y = (p.hq + p.ht - 1) / p.ht;
  }

  // 1x1 convolution over npx positions (any layout with channels last)
  void conv1x1(const float* in, int npx, const DevConv& w, const float* resid, int elu_acc, float* out_raw,
               float* out_elu) {
    ConvParams p{};
    p.in = in;
    p.in_n = 1; p.in_h = 1; p.in_w = npx; p.cin = w.cin;
    p.wgt = w.w; p.cout = w.cout; p.ntaps = 1; p.ntx = 1;
    p.ay0 = 0; p.ax0 = 0; p.ady = 1; p.adx = 1;
    p.n_img = 1; p.hq = 1; p.wq = npx; p.q0y = 0; p.q0x = 0;
    tile(p);
    p.bias = w.b; p.elu_acc = elu_acc;
    p.resid = resid; p.rh = 1; p.rw = npx; p.rsy = 1; p.rsx = 1;
    p.osy = 1; p.osx = 1; p.ory = 0; p.orx = 0; p.ho = 1; p.wo = npx; p.split = 0;
    p.out_raw = out_raw; p.out_elu = out_elu;
    p.split_tiles = (npx / nseq + 127) / 128;
    run(p);
  }

  // 3x3 convolution after causal_same_pad(x, {3, 3}, {1, 1})
  // (spectrostream.cpp:41-62: 2 rows on top, 1 column each side).
  // Residual at (oy / rsy, ox / rsx) of an (rh, rw) image.
  void conv3x3(Host4 in, const DevConv& w, const float* resid, int rh, int rw, int rsy, int rsx, int elu_acc,
               float* out_raw, float* out_elu, int split) {
    ConvParams p{};
    p.in = in.p;
    p.in_n = in.n; p.in_h = in.h; p.in_w = in.w; p.cin = in.c;
    p.wgt = w.w; p.cout = w.cout; p.ntaps = 9; p.ntx = 3;
    p.ay0 = -2; p.ax0 = -1; p.ady = 1; p.adx = 1;
    p.n_img = in.n; p.hq = in.h; p.wq = in.w; p.q0y = 0; p.q0x = 0;
    tile(p);
    p.bias = w.b; p.elu_acc = elu_acc;
    p.resid = resid; p.rh = rh; p.rw = rw; p.rsy = rsy; p.rsx = rsx;
    p.osy = 1; p.osx = 1; p.ory = 0; p.orx = 0; p.ho = in.h; p.wo = in.w; p.split = split;
    p.out_raw = out_raw; p.out_elu = out_elu;
    p.split_tiles = p.tiles_x * p.tiles_y * (in.n / nseq);
    run(p);
  }

  // One output phase (ry, rx) of a transposed convolution with stride
  // (sh, sw): full-size output row f = q_y sh + ry takes kernel rows
  // ry + sh j_y at input row q_y - j_y (likewise for columns); the block's
  // crop keeps rows [0, h sh) and columns [cws, cws + w sw).
  void convt_phase(Host4 in, const DevConv& w, const DecSpec& s, int ry, int rx, float* out) {
    const int cws = (s.tkw - s.sw) / 2;
    ConvParams p{};
    p.in = in.p;
    p.in_n = in.n; p.in_h = in.h; p.in_w = in.w; p.cin = in.c;
    p.wgt = w.w; p.cout = w.cout; p.ntaps = w.ntaps; p.ntx = w.ntx;
    p.ay0 = 0; p.ax0 = 0; p.ady = -1; p.adx = -1;
    p.n_img = in.n; p.hq = in.h; p.q0y = 0;
    p.q0x = ceil_div(cws - rx, s.sw);
    p.wq = floor_div(in.w * s.sw - 1 + cws - rx, s.sw) - p.q0x + 1;
    tile(p);
    p.bias = w.b; p.elu_acc = 1;
    p.resid = nullptr; p.rh = 0; p.rw = 0; p.rsy = 1; p.rsx = 1;
    p.osy = s.sh; p.osx = s.sw; p.ory = ry; p.orx = rx - cws; p.ho = in.h * s.sh; p.wo = in.w * s.sw; p.split = 0;
    p.out_raw = out; p.out_elu = nullptr;
    p.split_tiles = p.tiles_x * p.tiles_y * (in.n / nseq);
    run(p);
  }

  // decoder from x0 (B, S + 1, 1, 256) to spec (B, 4 S, 480, 4)
  void decoder(int B, int S) {
    nseq = B;
    const int Hs = S + 1, M0 = B * Hs;
    // input_proj: Res1x1Block 256 -> 2560 -> 2560, no pre-ELU (spectrostream.cpp:174-181)
    conv1x1(c->x0, M0, c->ip_sc, nullptr, 0, c->r, nullptr);
    conv1x1(c->x0, M0, c->ip_c1, nullptr, 1, c->y, nullptr);
    conv1x1(c->y, M0, c->ip_c2, c->r, 0, c->raw[0], c->elu);
    // unfold_width(x, 5) is a reshape: (B, Hs, 1, 2560) == (B, Hs, 5, 512)
    // input_conv: Res3x3Block 512, causal (spectrostream.cpp:191-199)
    const int W0 = kUnfold, C0 = kProj / kUnfold;
    conv3x3({c->elu, B, Hs, W0, C0}, c->ic_c1, nullptr, 0, 0, 1, 1, 1, c->y, nullptr, 0);
    conv3x3({c->y, B, Hs, W0, C0}, c->ic_c2, c->raw[0], Hs, W0, 1, 1, 0, c->raw[1], c->elu, 0);
    int cur = 1, n = B, h = Hs, w = W0, ch = C0;
    for (int i = 0; i < 7; ++i) {
      // DecoderResBlock (spectrostream.cpp:224-267)
      const DecSpec& s = kDec[i];
      const float* resid = c->raw[cur];
      if (c->has_sc[i]) {
        // shortcut(repeat(x)) == repeat(shortcut(x)): the 1x1 conv at the input resolution
        conv1x1(c->raw[cur], n * h * w, c->sc[i], nullptr, 0, c->r, nullptr);
        resid = c->r;
      }
      for (int ph = 0; ph < c->nphase[i]; ++ph)
        convt_phase({c->elu, n, h, w, ch}, c->ct[i][ph], s, c->phase_ry[i][ph], c->phase_rx[i][ph], c->y);
      const int ho = h * s.sh, wo = w * s.sw;
      const bool last = i == 6;
      const int split = i == 0 ? s.out / 2 : 0;  // stereo split after block 0 (spectrostream.cpp:385-392)
      conv3x3({c->y, n, ho, wo, s.out}, c->post[i], resid, h, w, s.sh, s.sw, 0, last ? nullptr : c->raw[1 - cur],
              c->elu, split);
      cur = 1 - cur;
      if (i == 0) {
        n *= 2;
        ch = s.out / 2;
      } else {
        ch = s.out;
      }
      h = ho;
      w = wo;
    }
    // elu -> output_conv 7x7 causal -> crop 4 rows -> stereo recombine
    ++kernels;
    need_act = std::max(need_act, (size_t)n * h * w * ch);
    if (launch) {
      OutConvParams o{c->elu, c->oc_w, c->oc_b, c->spec, B, h, w, kCrop};
      fail(launch_out_conv(o, c->s, pdl), "out_conv");
    }
  }

  void dequant(int B, int S, int levels, const int32_t* codes) {
    ++kernels;
    if (launch) {
      DequantParams d{codes, c->codebooks, c->x0, c->err, B, S, levels, c->C, c->D, 1};
      fail(launch_dequant(d, c->s, pdl), "dequant");
    }
  }

  void istft(int B, int frames, int target, const float* spec, float* audio) {
    kernels += 2;
    need_act = std::max(need_act, (size_t)B * 2 * frames * kFft);  // windowed frames in the y buffer
    if (launch) {
      IstftParams q{spec, c->synth, c->cosv, audio, c->y, B, frames, target};
      fail(launch_istft(q, c->s, pdl), "istft");
    }
  }
};

void check_sizes(mrtss_codec* c, int B, int S) {
  if (B <= 0 || S <= 0) throw Error{MRTDF_ERR_INVALID, "B and S must be positive"};
  if (B > c->max_batch || S > c->max_frames)
    throw Error{MRTDF_ERR_RANGE, "B = " + std::to_string(B) + ", S = " + std::to_string(S) +
                                     " exceed the codec's capacity (" + std::to_string(c->max_batch) + ", " +
                                     std::to_string(c->max_frames) + ")"};
}

void require_loaded(mrtss_codec* c) {
  if (!c) throw Error{MRTDF_ERR_INVALID, "NULL codec"};
  if (!c->loaded) throw Error{MRTDF_ERR_STATE, "load the codec's weights first"};
}

// Read and clear the device error word after a synchronise.
void sync_and_check(mrtss_codec* c) {
  SS_CUDA(cudaStreamSynchronize(c->s));
  int e = 0;
  SS_CUDA(cudaMemcpy(&e, c->err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e) {
    SS_CUDA(cudaMemset(c->err, 0, sizeof(int)));
    if (e & kErrMbarTimeout) throw Error{MRTDF_ERR_TIMEOUT, "codec: a device-side bounded wait gave up"};
    if (e & kErrBadToken) throw Error{MRTDF_ERR_RANGE, "codec: an RVQ code outside [0, codebook size)"};
    throw Error{MRTDF_ERR_CUDA, "codec: device error word " + std::to_string(e)};
  }
}

// Canonical host tensors -> device layouts; `get` returns float32 data of a key.
void upload(mrtss_codec* c, const std::function<const float*(const std::string&, const std::vector<int64_t>&)>& get,
            const float* codebooks, int K, int Cb, int D) {
  if (D != kEmb) throw Error{MRTDF_ERR_INVALID, "codebooks must have D = 256"};
  if (K <= 0 || Cb <= 0) throw Error{MRTDF_ERR_INVALID, "codebooks must be (K, C, 256) with K, C > 0"};
  std::vector<float> host;  // all weights back to back, 64-byte aligned pieces
  struct Piece {
    size_t off;
    float** dst;
  };
  std::vector<Piece> pieces;
  auto add = [&](const std::vector<float>& v, float** dst) {
    host.resize((host.size() + 15) & ~size_t(15));
    pieces.push_back({host.size(), dst});
    host.insert(host.end(), v.begin(), v.end());
  };
  auto bias = [&](const std::string& p, int O, float** dst) {
    const float* b = get(p + ".bias", {O});
    add(std::vector<float>(b, b + O), dst);
  };
  // conv (O, I, kh, kw) -> (O, kh * kw, I)
  auto conv = [&](const std::string& p, int O, int I, int kh, int kw, DevConv& d) {
    const float* w = get(p + ".weight", {O, I, kh, kw});
    std::vector<float> t((size_t)O * kh * kw * I);
    for (int o = 0; o < O; ++o)
      for (int i = 0; i < I; ++i)
        for (int y = 0; y < kh; ++y)
          for (int x = 0; x < kw; ++x)
            t[(((size_t)o * kh + y) * kw + x) * I + i] = w[(((size_t)o * I + i) * kh + y) * kw + x];
    d.cout = O; d.cin = I; d.ntaps = kh * kw; d.ntx = kw;
    add(t, &d.w);
    bias(p, O, &d.b);
  };
  conv("input_proj.conv1", kProj, kEmb, 1, 1, c->ip_c1);
  conv("input_proj.conv2", kProj, kProj, 1, 1, c->ip_c2);
  conv("input_proj.shortcut", kProj, kEmb, 1, 1, c->ip_sc);
  conv("input_conv.conv1", 512, 512, 3, 3, c->ic_c1);
  conv("input_conv.conv2", 512, 512, 3, 3, c->ic_c2);
  for (int i = 0; i < 7; ++i) {
    const DecSpec& s = kDec[i];
    const std::string p = "decoder_blocks." + std::to_string(i);
    // transposed conv (I, O, kh, kw) -> one (O, taps, I) matrix per output
    // phase (ry, rx): tap (jy, jx) holds kernel element (ry + sh jy, rx + sw jx)
    const float* w = get(p + ".conv_transpose.weight", {s.in, s.out, s.tkh, s.tkw});
    c->nphase[i] = 0;
    for (int ry = 0; ry < s.sh; ++ry)
      for (int rx = 0; rx < s.sw; ++rx) {
        const int nty = (s.tkh - ry + s.sh - 1) / s.sh, ntx = (s.tkw - rx + s.sw - 1) / s.sw;
        DevConv& d = c->ct[i][c->nphase[i]];
        c->phase_ry[i][c->nphase[i]] = ry;
        c->phase_rx[i][c->nphase[i]] = rx;
        ++c->nphase[i];
        std::vector<float> t((size_t)s.out * nty * ntx * s.in);
        for (int o = 0; o < s.out; ++o)
          for (int jy = 0; jy < nty; ++jy)
            for (int jx = 0; jx < ntx; ++jx)
              for (int ii = 0; ii < s.in; ++ii)
                t[(((size_t)o * nty + jy) * ntx + jx) * s.in + ii] =
                    w[(((size_t)ii * s.out + o) * s.tkh + ry + s.sh * jy) * s.tkw + rx + s.sw * jx];
        d.cout = s.out; d.cin = s.in; d.ntaps = nty * ntx; d.ntx = ntx;
        add(t, &d.w);
        bias(p + ".conv_transpose", s.out, &d.b);
      }
    conv(p + ".conv", s.out, s.out, 3, 3, c->post[i]);
    c->has_sc[i] = s.in != s.out;
    if (c->has_sc[i]) conv(p + ".shortcut", s.out, s.in, 1, 1, c->sc[i]);
  }
  {
    // output_conv (2, 64, 7, 7) -> (2, 7, 7, 64)
    const float* w = get("output_conv.weight", {2, kOutCh, 7, 7});
    std::vector<float> t((size_t)2 * 49 * kOutCh);
    for (int o = 0; o < 2; ++o)
      for (int i = 0; i < kOutCh; ++i)
        for (int y = 0; y < 7; ++y)
          for (int x = 0; x < 7; ++x) t[((o * 7 + y) * 7 + x) * kOutCh + i] = w[((o * kOutCh + i) * 7 + y) * 7 + x];
    add(t, &c->oc_w);
    bias("output_conv", 2, &c->oc_b);
  }
  add(std::vector<float>(codebooks, codebooks + (size_t)K * Cb * D), &c->codebooks);
  {
    // synthesis window (periodic Hann / sum of squares over the two hops) in
    // float like istft_postprocess; cosine table for the inverse DFT
    std::vector<float> win(kFft), synth(kFft), cosv(kFft);
    const float two_pi_over_n = 2.0f * static_cast<float>(M_PI) / static_cast<float>(kFft);
    for (int t = 0; t < kFft; ++t) win[t] = 0.5f - 0.5f * std::cos(static_cast<float>(t) * two_pi_over_n);
    for (int j = 0; j < kHop; ++j) {
      const float p = win[j] * win[j] + win[j + kHop] * win[j + kHop];
      synth[j] = win[j] / p;
      synth[j + kHop] = win[j + kHop] / p;
    }
    for (int m = 0; m < kFft; ++m) cosv[m] = (float)std::cos(2.0 * M_PI * m / kFft);
    add(synth, &c->synth);
    add(cosv, &c->cosv);
  }
  if (c->weights) {
    SS_CUDA(cudaFree(c->weights));
    c->weights = nullptr;
  }
  for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
  c->graphs.clear();
  SS_CUDA(cudaMalloc(&c->weights, host.size() * sizeof(float)));
  SS_CUDA(cudaMemcpy(c->weights, host.data(), host.size() * sizeof(float), cudaMemcpyHostToDevice));
  for (const Piece& p : pieces) *p.dst = reinterpret_cast<float*>(c->weights) + p.off;
  c->K = K;
  c->C = Cb;
  c->D = D;
  c->loaded = true;
}

void fill_codec_random(uint64_t seed, int levels, std::map<std::string, std::vector<float>>& out,
                       std::vector<float>& codebooks) {
  const auto specs = codec_specs();
  for (size_t i = 0; i < specs.size(); ++i) {
    int64_t n = 1;
    for (auto d : specs[i].shape) n *= d;
    std::vector<float> v((size_t)n);
    fill_random_tensor(seed, (int)i, specs[i].stddev, false, false, v.data(), n);
    out[specs[i].key] = std::move(v);
  }
  codebooks.resize((size_t)levels * kCodebookSize * kEmb);
  fill_random_tensor(seed, 1000, 0.25f, false, false, codebooks.data(), (int64_t)codebooks.size());
}

cudaGraphExec_t decode_graph(mrtss_codec* c, int B, int S, int levels) {
  const std::array<int, 3> key{B, S, levels};
  auto it = c->graphs.find(key);
  if (it != c->graphs.end()) return it->second;
  SS_CUDA(cudaStreamBeginCapture(c->s, cudaStreamCaptureModeThreadLocal));
  try {
    Plan p{c, true};
    p.dequant(B, S, levels, c->codes);
    p.decoder(B, S);
    p.istft(B, 4 * S, S * MRTSS_FRAME_SAMPLES, c->spec, c->audio);
  } catch (...) {
    cudaGraph_t g = nullptr;
    cudaStreamEndCapture(c->s, &g);
    if (g) cudaGraphDestroy(g);
    throw;
  }
  cudaGraph_t g = nullptr;
  SS_CUDA(cudaStreamEndCapture(c->s, &g));
  cudaGraphExec_t ge = nullptr;
  const cudaError_t e = cudaGraphInstantiate(&ge, g, 0);
  cudaGraphDestroy(g);
  SS_CUDA(e);
  c->graphs[key] = ge;
  return ge;
}

void check_codes(mrtss_codec* c, const int32_t* codes, size_t n, int levels) {
  if (levels <= 0 || levels > c->K)
    throw Error{MRTDF_ERR_INVALID, "levels must be in [1, " + std::to_string(c->K) + "]"};
  for (size_t i = 0; i < n; ++i)
    if (codes[i] < 0 || codes[i] >= c->C)
      throw Error{MRTDF_ERR_RANGE, "code " + std::to_string(codes[i]) + " at " + std::to_string(i) +
                                       " outside [0, " + std::to_string(c->C) + ")"};
}

}  // namespace

extern "C" {

int mrtss_write_random_safetensors(uint64_t seed, int levels, const char* decoder_path, const char* codebooks_path) {
  return guarded([&] {
    if (!decoder_path || !codebooks_path) throw Error{MRTDF_ERR_INVALID, "NULL path"};
    if (levels <= 0) throw Error{MRTDF_ERR_INVALID, "levels must be positive"};
    std::map<std::string, std::vector<float>> w;
    std::vector<float> cb;
    fill_codec_random(seed, levels, w, cb);
    std::vector<OutTensor> out;
    for (const auto& s : codec_specs()) out.push_back({s.key, s.shape, w[s.key].data()});
    write_safetensors(decoder_path, out);
    write_safetensors(codebooks_path, {{"codebooks", {levels, kCodebookSize, kEmb}, cb.data()}});
  });
}

int mrtss_create(int device, int max_batch, int max_frames, mrtss_codec** out) {
  return guarded([&] {
    if (!out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    *out = nullptr;
    if (max_batch <= 0 || max_frames <= 0) throw Error{MRTDF_ERR_INVALID, "capacities must be positive"};
    SS_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    SS_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
      throw Error{MRTDF_ERR_CUDA, std::string("the codec needs an sm_100 (B200) device, found ") + prop.name};
    std::unique_ptr<mrtss_codec> c(new mrtss_codec());
    c->device = device;
    c->max_batch = max_batch;
    c->max_frames = max_frames;
    for (int i = 0; i < 7; ++i) {  // block structure (the weights fill the rest at load)
      c->has_sc[i] = kDec[i].in != kDec[i].out;
      c->nphase[i] = 0;
      for (int ry = 0; ry < kDec[i].sh; ++ry)
        for (int rx = 0; rx < kDec[i].sw; ++rx) {
          c->phase_ry[i][c->nphase[i]] = ry;
          c->phase_rx[i][c->nphase[i]] = rx;
          ++c->nphase[i];
        }
    }
    SS_CUDA(cudaStreamCreateWithFlags(&c->s, cudaStreamNonBlocking));
    SS_CUDA(conv_tc_set_smem_limits());
    // buffer sizes from a dry walk of the plan at full capacity
    Plan p{c.get(), false};
    p.decoder(max_batch, max_frames);
    c->act_floats = p.need_act;
    c->x0_floats = (size_t)max_batch * (max_frames + 1) * kEmb;
    c->spec_floats = (size_t)max_batch * 4 * max_frames * MRTSS_STFT_BINS * 4;
    c->audio_floats = (size_t)max_batch * max_frames * MRTSS_FRAME_SAMPLES * 2;
    c->codes_ints = (size_t)max_batch * max_frames * 64;  // up to 64 RVQ levels
    auto alloc = [&](size_t bytes) {
      void* q = nullptr;
      SS_CUDA(cudaMalloc(&q, bytes));
      c->allocs.push_back(q);
      return q;
    };
    c->x0 = (float*)alloc(c->x0_floats * 4);
    c->raw[0] = (float*)alloc(c->act_floats * 4);
    c->raw[1] = (float*)alloc(c->act_floats * 4);
    c->elu = (float*)alloc(c->act_floats * 4);
    c->y = (float*)alloc(c->act_floats * 4);
    c->r = (float*)alloc(c->act_floats * 4);
    c->spec = (float*)alloc(c->spec_floats * 4);
    c->audio = (float*)alloc(c->audio_floats * 4);
    c->codes = (int32_t*)alloc(c->codes_ints * 4);
    c->err = (int*)alloc(sizeof(int));
    SS_CUDA(cudaMemset(c->err, 0, sizeof(int)));
    *out = c.release();
  });
}

void mrtss_destroy(mrtss_codec* c) { delete c; }

int mrtss_load_safetensors(mrtss_codec* c, const char* decoder_path, const char* codebooks_path) {
  return guarded([&] {
    if (!c || !decoder_path || !codebooks_path) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    SS_CUDA(cudaSetDevice(c->device));
    SafetensorsFile f(decoder_path);
    SafetensorsFile fc(codebooks_path);
    std::map<std::string, std::vector<float>> conv;
    auto as_f32 = [&](const TensorRef* t, const std::string& key) -> const float* {
      if (t->dtype == "F32") return reinterpret_cast<const float*>(t->data);
      if (t->dtype != "BF16") throw Error{MRTDF_ERR_INVALID, "unsupported dtype " + t->dtype + " for " + key};
      auto& v = conv[key];
      v.resize((size_t)t->numel());
      const uint16_t* s = reinterpret_cast<const uint16_t*>(t->data);
      for (int64_t i = 0; i < t->numel(); ++i) {
        const uint32_t u = (uint32_t)s[i] << 16;
        std::memcpy(&v[(size_t)i], &u, 4);
      }
      return v.data();
    };
    auto get = [&](const std::string& key, const std::vector<int64_t>& shape) -> const float* {
      const TensorRef* t = f.find(key);
      if (!t) throw Error{MRTDF_ERR_KEY, "WeightBundle " + std::string(decoder_path) + ": missing key \"" + key + "\""};
      if (t->shape != shape) throw Error{MRTDF_ERR_INVALID, "shape mismatch for " + key};
      return as_f32(t, key);
    };
    const TensorRef* cb = fc.find("codebooks");
    if (!cb) throw Error{MRTDF_ERR_KEY, "WeightBundle " + std::string(codebooks_path) + ": missing key \"codebooks\""};
    if (cb->shape.size() != 3) throw Error{MRTDF_ERR_INVALID, "codebooks must be (K, C, D)"};
    upload(c, get, as_f32(cb, "codebooks"), (int)cb->shape[0], (int)cb->shape[1], (int)cb->shape[2]);
  });
}

int mrtss_load_random(mrtss_codec* c, uint64_t seed, int levels) {
  return guarded([&] {
    if (!c) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (levels <= 0) throw Error{MRTDF_ERR_INVALID, "levels must be positive"};
    SS_CUDA(cudaSetDevice(c->device));
    std::map<std::string, std::vector<float>> w;
    std::vector<float> cb;
    fill_codec_random(seed, levels, w, cb);
    auto get = [&](const std::string& key, const std::vector<int64_t>&) -> const float* {
      auto it = w.find(key);
      if (it == w.end()) throw Error{MRTDF_ERR_KEY, "missing key \"" + key + "\""};
      return it->second.data();
    };
    upload(c, get, cb.data(), levels, kCodebookSize, kEmb);
  });
}

int mrtss_rvq_dequantize(mrtss_codec* c, const int32_t* codes, int n, int levels, float* out) {
  return guarded([&] {
    require_loaded(c);
    if (!codes || !out || n <= 0) throw Error{MRTDF_ERR_INVALID, "bad arguments"};
    SS_CUDA(cudaSetDevice(c->device));
    check_codes(c, codes, (size_t)n * levels, levels);
    if ((size_t)n * levels > c->codes_ints || (size_t)n * kEmb > c->x0_floats)
      throw Error{MRTDF_ERR_RANGE, "n exceeds the codec's capacity"};
    SS_CUDA(cudaMemcpyAsync(c->codes, codes, (size_t)n * levels * 4, cudaMemcpyHostToDevice, c->s));
    Plan p{c, true, false};
    DequantParams d{c->codes, c->codebooks, c->x0, c->err, 1, n, levels, c->C, c->D, 0};
    p.fail(launch_dequant(d, c->s, false), "dequant");
    SS_CUDA(cudaMemcpyAsync(out, c->x0, (size_t)n * kEmb * 4, cudaMemcpyDeviceToHost, c->s));
    sync_and_check(c);
  });
}

int mrtss_decode(mrtss_codec* c, const float* emb, int B, int S, float* spec) {
  return guarded([&] {
    require_loaded(c);
    if (!emb || !spec) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    check_sizes(c, B, S);
    SS_CUDA(cudaSetDevice(c->device));
    // (B, S, 256) -> (B, S + 1, 256) with the appended zero frame (spectrostream.cpp:372-374)
    SS_CUDA(cudaMemsetAsync(c->x0, 0, (size_t)B * (S + 1) * kEmb * 4, c->s));
    SS_CUDA(cudaMemcpy2DAsync(c->x0, (size_t)(S + 1) * kEmb * 4, emb, (size_t)S * kEmb * 4, (size_t)S * kEmb * 4, B,
                              cudaMemcpyHostToDevice, c->s));
    Plan p{c, true, false};
    p.decoder(B, S);
    SS_CUDA(cudaMemcpyAsync(spec, c->spec, (size_t)B * 4 * S * MRTSS_STFT_BINS * 4 * 4, cudaMemcpyDeviceToHost, c->s));
    sync_and_check(c);
  });
}

int mrtss_istft(mrtss_codec* c, const float* spec, int B, int frames, int target, float* audio) {
  return guarded([&] {
    if (!c || !spec || !audio) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (B <= 0 || frames <= 0 || target <= 0 || target > (frames + 1) * kHop)
      throw Error{MRTDF_ERR_INVALID, "need B, frames > 0 and 0 < target <= (frames + 1) * 480"};
    if ((size_t)B * frames * MRTSS_STFT_BINS * 4 > c->spec_floats || (size_t)B * target * 2 > c->audio_floats ||
        (size_t)B * 2 * frames * kFft > c->act_floats)
      throw Error{MRTDF_ERR_RANGE, "spectrogram or audio exceeds the codec's capacity"};
    if (!c->synth) throw Error{MRTDF_ERR_STATE, "load the codec's weights first"};
    SS_CUDA(cudaSetDevice(c->device));
    SS_CUDA(cudaMemcpyAsync(c->spec, spec, (size_t)B * frames * MRTSS_STFT_BINS * 4 * 4, cudaMemcpyHostToDevice, c->s));
    Plan p{c, true, false};
    p.istft(B, frames, target, c->spec, c->audio);
    SS_CUDA(cudaMemcpyAsync(audio, c->audio, (size_t)B * target * 2 * 4, cudaMemcpyDeviceToHost, c->s));
    sync_and_check(c);
  });
}

int mrtss_decode_tokens(mrtss_codec* c, const int32_t* codes, int B, int S, int levels, float* audio) {
  return guarded([&] {
    require_loaded(c);
    if (!codes || !audio) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    check_sizes(c, B, S);
    check_codes(c, codes, (size_t)B * S * levels, levels);
    if ((size_t)B * S * levels > c->codes_ints) throw Error{MRTDF_ERR_RANGE, "too many RVQ levels"};
    SS_CUDA(cudaSetDevice(c->device));
    SS_CUDA(cudaMemcpyAsync(c->codes, codes, (size_t)B * S * levels * 4, cudaMemcpyHostToDevice, c->s));
    SS_CUDA(cudaGraphLaunch(decode_graph(c, B, S, levels), c->s));
    SS_CUDA(cudaMemcpyAsync(audio, c->audio, (size_t)B * S * MRTSS_FRAME_SAMPLES * 2 * 4, cudaMemcpyDeviceToHost,
                            c->s));
    sync_and_check(c);
  });
}

int mrtss_decode_tokens_dev(mrtss_codec* c, const int32_t* codes_dev, int B, int S, int levels, float* audio_dev) {
  return guarded([&] {
    require_loaded(c);
    if (!codes_dev || !audio_dev) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    check_sizes(c, B, S);
    if (levels <= 0 || levels > c->K) throw Error{MRTDF_ERR_INVALID, "levels out of range"};
    if ((size_t)B * S * levels > c->codes_ints) throw Error{MRTDF_ERR_RANGE, "too many RVQ levels"};
    SS_CUDA(cudaSetDevice(c->device));
    SS_CUDA(cudaMemcpyAsync(c->codes, codes_dev, (size_t)B * S * levels * 4, cudaMemcpyDeviceToDevice, c->s));
    SS_CUDA(cudaGraphLaunch(decode_graph(c, B, S, levels), c->s));
    SS_CUDA(cudaMemcpyAsync(audio_dev, c->audio, (size_t)B * S * MRTSS_FRAME_SAMPLES * 2 * 4,
                            cudaMemcpyDeviceToDevice, c->s));
  });
}

int mrtss_sync(mrtss_codec* c) {
  return guarded([&] {
    if (!c) throw Error{MRTDF_ERR_INVALID, "NULL codec"};
    SS_CUDA(cudaSetDevice(c->device));
    sync_and_check(c);
  });
}

void* mrtss_cuda_stream(mrtss_codec* c) { return c ? (void*)c->s : nullptr; }

long long mrtss_decode_kernels(mrtss_codec* c, int B, int S) {
  if (!c || B <= 0 || S <= 0) return -1;
  Plan p{c, false};
  p.dequant(B, S, 1, nullptr);
  p.decoder(B, S);
  p.istft(B, 4 * S, S * MRTSS_FRAME_SAMPLES, nullptr, nullptr);
  return p.kernels;
}

}  // extern "C"

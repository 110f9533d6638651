// SpectroStream codec decode phase on the device: RVQ dequantisation, the
// decoder's convolutions as implicit GEMMs on the tensor cores (tf32
// operands, fp32 accumulation in tensor memory), the 7x7 output convolution
// and the iSTFT. Activations are NHWC float32, like the reference's float32
// decoder (system.cpp:118-119).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mrtdf {

// One convolution (or one output phase of a transposed convolution) as an
// implicit GEMM: rows = output positions q of a (hq x wq) grid per image,
// columns = output channels, K = taps x cin. Tap t = (ty, tx) = (t / ntx,
// t % ntx) reads the input at (q_y + ay0 + ty * ady, q_x + ax0 + tx * adx);
// reads outside the input are zero (the convolution's padding).
struct ConvParams {
  // A operand (input activation, NHWC float32) and its extent
  const float* in;
  int in_n, in_h, in_w, cin;
  // B operand: weights (cout, ntaps, cin) row-major
  const float* wgt;
  int cout, ntaps, ntx;
  int ay0, ax0, ady, adx;
  // output-position grid and its tiling (wt x ht positions per 128-row tile)
  int n_img, hq, wq, q0y, q0x, wt, ht, tiles_x, tiles_y;
  // epilogue: value = acc + bias[n]; if elu_acc the value becomes elu(value);
  // then + resid[img, oy / rsy, ox / rsx, n] when resid is set. Position q
  // goes to output pixel (q_y * osy + ory, q_x * osx + orx) of an (ho, wo)
  // image, skipped when outside. out_raw receives the value, out_elu
  // elu(value) (either may be null). split > 0: column n goes to image
  // (n / split) * n_img + img, channel n % split (the decoder's stereo split).
  const float* bias;
  int elu_acc;
  const float* resid;
  int rh, rw, rsy, rsx;
  int osy, osx, ory, orx, ho, wo, split;
  float* out_raw;
  float* out_elu;
  // M tiles of this layer for ONE sequence: the split-K factor derives from
  // it, so results do not depend on the batch size (0 = the grid's tiles)
  int split_tiles;
};

// Output convolution 7x7 (64 -> 2, causal padding) fused with the temporal
// crop of the first `crop` rows and the stereo recombine:
// in (2 B, H, W, 64) elu'd activations -> spec (B, H - crop, W, 4).
struct OutConvParams {
  const float* in;
  const float* wgt;   // (2, 7, 7, 64)
  const float* bias;  // (2)
  float* spec;
  int B, H, W, crop;
};

struct IstftParams {
  const float* spec;   // (B, frames, 480, 4)
  const float* synth;  // (960) synthesis window
  const float* cosv;   // (960) cos(2 pi m / 960)
  float* audio;        // (B, target, 2)
  float* frames_buf;   // scratch (B, 2, frames, 960): windowed frames
  int B, frames, target;
};

struct DequantParams {
  const int32_t* codes;     // (B, S, levels)
  const float* codebooks;   // (K, C, D)
  float* out;               // (B, S + pad_frames, 1, D): rows >= S are zero
  int* err;
  int B, S, levels, C, D, pad_frames;
};

constexpr int kConvBK = 32;  // fp32 elements per 128-byte operand row
cudaError_t launch_conv_tc(const ConvParams& p, int* err, cudaStream_t s, bool pdl);
cudaError_t conv_tc_set_smem_limits();
cudaError_t launch_out_conv(const OutConvParams& p, cudaStream_t s, bool pdl);
// two launches: windowed frames, then overlap-add
cudaError_t launch_istft(const IstftParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_dequant(const DequantParams& p, cudaStream_t s, bool pdl);

}  // namespace mrtdf

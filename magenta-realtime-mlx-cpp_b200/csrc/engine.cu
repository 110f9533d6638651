// Engine and C ABI (include/mrtdf.h): weight upload into fused device
// layouts, per-stream KV arenas, the step sequences of encode /
// temporal_step / depth_step / sample, and the whole-chunk CUDA graph of
// generate_tokens.
//
// Reference call structure (rhymeswithlion/magenta-realtime-mlx-cpp):
//   Depthformer ctor       depthformer/model.cpp:173-213
//   encode                 model.cpp:226-241
//   temporal_step (eager)  model.cpp:322-514 (493-513)
//   depth_step (eager)     model.cpp:516-659 (638-659)
//   bias precompute        model.cpp:302-320
//   generate_tokens        depthformer/decode.cpp:239-573 (non-speculative)
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/mrtdf.h"
#include "decode_kernels.cuh"
#include "glue_kernels.cuh"
#include "device_errors.h"
#include "encoder_kernels.cuh"
#include "fused_decode.cuh"
#include "host_util.h"

using namespace mrtdf;

namespace {

#define CUDA_OK(expr)                                                                                    \
  do {                                                                                                   \
    cudaError_t e_ = (expr);                                                                             \
    if (e_ != cudaSuccess)                                                                               \
      throw Error{MRTDF_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)};                   \
  } while (0)

bool env_flag(const char* name, bool dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  return !(v[0] == '0' || v[0] == 'n' || v[0] == 'N' || v[0] == 'f' || v[0] == 'F');
}

// Sub-allocator over one cudaMalloc: 256-byte aligned slices.
struct Arena {
  uint8_t* base = nullptr;
  size_t cap = 0, used = 0;
  void reserve(size_t bytes) {
    if (base) cudaFree(base);
    base = nullptr;
    cap = bytes;
    used = 0;
    if (bytes) CUDA_OK(cudaMalloc(&base, bytes));
  }
  void* take(size_t bytes) {
    const size_t off = (used + 255) & ~(size_t)255;
    if (off + bytes > cap) throw Error{MRTDF_ERR_CUDA, "arena overflow"};
    used = off + bytes;
    return base + off;
  }
  ~Arena() {
    if (base) cudaFree(base);
  }
};

struct EncLayerDev {
  void *wqkv, *wo, *n_attn, *wi, *wout, *n_ffn;
};
struct DecLayerDev {
  void *wqkv, *wo, *n_self, *wcq, *wco, *n_cross, *wi, *wout, *n_ffn;
  // copies for the fused phases (bf16): o_proj / cross o_proj as
  // [H][d][64 + 8 pad], wo as [nclusters][d][Uc + 8 pad]; q/k/v, cross q
  // and wi rows with a 16-byte pad after each row (one TMA copy per CTA)
  void *wo_blk = nullptr, *wco_blk = nullptr, *wout_blk = nullptr;
  void *wqkv_pad = nullptr, *wcq_pad = nullptr, *wi_pad = nullptr;
};

// A hidden state between decode phases: `x` itself, or (fused phases)
// R(x + R(acc / 2^32)) with x the residual stream and acc the split sums.
struct Hidden {
  const void* x;
  const long long* acc;
};

}  // namespace

struct mrtdf_engine {
  mrtdf_config c{};
  int device = 0;
  int num_sms = 148;
  int esize = 2;  // bytes per element of the compute dtype
  bool loaded = false;
  bool pdl = true;
  // bf16 decode self-attention inside a thread-block cluster per head that
  // also computes the head's q/k/v rows (MRTDF_CLUSTER_ATTN=0: separate kernel)
  bool cluster_attn = true;
  // wide streams: largest split-K cluster of the tcgen05 decode GEMMs
  // (MRTDF_WIDE_KSPLIT; 64 CFG pairs: 607 ms per chunk unsplit, 504 ms at 8)
  int wide_ksplit = 8;
  // fused decode phases for streams of at most two bf16 rows (one CFG pair)
  bool fused = false;
  FfnPlan ffn_plan;
  Arena weights;
  void* emb = nullptr;
  void* enc_norm = nullptr;
  void* dec_norm = nullptr;
  void* lm_head = nullptr;
  void* wckv = nullptr;  // (Lt * 2 * inner, d)
  std::vector<EncLayerDev> enc;
  std::vector<DecLayerDev> tl, dl;
  float* tbias = nullptr;  // (Tmax, H, Tmax)
  float* dbias = nullptr;  // (depth, H, depth)
  float* pe = nullptr;     // (Smax, d)
  int inner() const { return c.num_heads * c.d_kv; }
};

struct GraphKey {
  int frames, depth, top_k, masked, has_uniforms, seq_len;
  float temperature, w;
  bool operator<(const GraphKey& o) const {
    return std::memcmp(this, &o, sizeof(GraphKey)) < 0;
  }
};

struct mrtdf_stream {
  mrtdf_engine* eng = nullptr;
  int nseq = 1, rps = 2, B = 2;
  cudaStream_t s = nullptr;
  Arena mem;
  // activations (compute dtype unless noted)
  void *tx, *dx, *tin, *din, *fsum, *qb, *ao, *hb;
  float* logits;  // (B, V)
  float* stage_f32;  // host<->device float staging, (B, max(d, V))
  // caches
  void *tk, *tv, *ck, *cv, *dk, *dv;
  // encoder scratch
  void *ex, *en, *eqkv, *eo, *eh;
  void* xn;  // (B, d) normalised rows of the wide decode path
  // fused phases: three int64 accumulators (B, d) in a rotation, two bf16
  // residual buffers (B, d), and their ring positions
  bool fused = false;
  long long* facc = nullptr;
  void* fx[2] = {nullptr, nullptr};
  int fk = 0, fj = 0;
  int32_t* ids;
  int32_t* tokens;  // (nseq, Tmax, depth)
  uint64_t* seeds;  // (nseq)
  int32_t* forced;  // (nseq)
  int* err;
  float* uniforms = nullptr;
  size_t uniforms_cap = 0;
  uint64_t* seed_table = nullptr;  // per-chunk seeds of mrtdf_generate_stream_dev
  size_t seed_table_cap = 0;
  // host state
  bool encoded = false;
  int S = 0;
  int t_len = 0, d_len = 0;
  bool have_temporal = false;
  std::map<GraphKey, cudaGraphExec_t> graphs;
  std::map<GraphKey, long long> graph_kernels;  // kernel nodes of each chunk graph
  long long last_chunk_kernels = 0;              // of the chunk run last (graph or stream launches)
  // measurement hook: when set, only the GEMV phases are enqueued and their
  // launches / algorithmic bytes are counted
  // measurement hook: when set, only the weight-streaming decode phases of
  // the selected stacks (bit 0 temporal, bit 1 depth + lm_head) are
  // enqueued and their launches / algorithmic bytes are counted
  bool gemv_only = false;
  int phase_mask = 3;
  bool in_depth = false;
  long long gemv_launches = 0;
  double gemv_bytes = 0.0;
  ~mrtdf_stream() {
    for (auto& kv : graphs) cudaGraphExecDestroy(kv.second);
    if (s) cudaStreamDestroy(s);
  }
};

// ---------------------------------------------------------------------------
// helpers
// ---------------------------------------------------------------------------
namespace {


void check_cuda(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw Error{MRTDF_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e)};
}

// Convert host float32 data to the compute dtype's bytes.
std::vector<uint8_t> to_dtype(const float* src, size_t n, int dtype) {
  std::vector<uint8_t> out(n * (dtype == MRTDF_DTYPE_BF16 ? 2 : 4));
  if (dtype == MRTDF_DTYPE_BF16) {
    uint16_t* o = (uint16_t*)out.data();
    parallel_for((int64_t)n, [&](int64_t a, int64_t b) {
      for (int64_t i = a; i < b; ++i) o[i] = bf16_bits(src[i]);
    });
  } else {
    std::memcpy(out.data(), src, n * 4);
  }
  return out;
}

// Weight source: key -> float32 host data.
struct WeightSource {
  std::function<const float*(const std::string&, int64_t)> get;
};

}  // namespace

// Upload every weight into fused device tensors.
static void upload_weights(mrtdf_engine* E, const WeightSource& src) {
  const mrtdf_config& c = E->c;
  const int64_t d = c.d_model, in = E->inner(), ff = c.d_ff, V = c.vocab_size;
  const int es = E->esize;
  // bytes: count everything first
  size_t total = 0;
  auto add = [&](int64_t n) { total += ((size_t)n * es + 255) & ~(size_t)255; };
  add(V * d);
  for (int i = 0; i < c.num_encoder_layers; ++i) {
    add(3 * in * d); add(d * in); add(d); add(2 * ff * d); add(d * ff); add(d);
  }
  add(d);
  for (int i = 0; i < c.num_temporal_layers; ++i) {
    add(3 * in * d); add(d * in); add(d); add(in * d); add(d * in); add(d); add(2 * ff * d); add(d * ff); add(d);
  }
  add((int64_t)c.num_temporal_layers * 2 * in * d);
  for (int i = 0; i < c.num_depth_layers; ++i) {
    add(3 * in * d); add(d * in); add(d); add(2 * ff * d); add(d * ff); add(d);
  }
  add(d);
  add(V * d);
  const size_t tb = (size_t)c.max_frames * c.num_heads * c.max_frames * 4;
  const size_t db = (size_t)c.rvq_depth * c.num_heads * c.rvq_depth * 4;
  const size_t pb = (size_t)c.max_encoder_length * d * 4;
  if (E->fused) {
    const int64_t blk = (int64_t)c.num_heads * d * 72;                                 // o_proj block elements
    const int64_t oblk = (int64_t)E->ffn_plan.nclusters * d * (E->ffn_plan.Uc + 8);  // wo block elements
    const int64_t rp = d + 8;  // padded row elements
    for (int i = 0; i < c.num_temporal_layers; ++i) {
      add(blk); add(blk); add(oblk); add(3 * in * rp); add(in * rp); add(2 * ff * rp);
    }
    for (int i = 0; i < c.num_depth_layers; ++i) { add(blk); add(oblk); add(3 * in * rp); add(2 * ff * rp); }
  }
  total += tb + db + pb + 3 * 256;
  E->weights.reserve(total);

  std::vector<float> tmp;
  auto put = [&](void* dst, const float* host, int64_t n) {
    std::vector<uint8_t> bytes = to_dtype(host, (size_t)n, c.dtype);
    CUDA_OK(cudaMemcpy(dst, bytes.data(), bytes.size(), cudaMemcpyHostToDevice));
  };
  auto fetch = [&](const std::string& key, int64_t n) { return src.get(key, n); };
  auto single = [&](const std::string& key, int64_t n) {
    void* dst = E->weights.take((size_t)n * es);
    put(dst, fetch(key, n), n);
    return dst;
  };
  // concatenate rows of several (rows_i, d) matrices
  auto concat = [&](const std::vector<std::pair<std::string, int64_t>>& parts, int64_t cols) {
    int64_t rows = 0;
    for (auto& p : parts) rows += p.second;
    tmp.resize((size_t)(rows * cols));
    int64_t r = 0;
    for (auto& p : parts) {
      const float* h = fetch(p.first, p.second * cols);
      std::memcpy(&tmp[(size_t)(r * cols)], h, (size_t)(p.second * cols) * 4);
      r += p.second;
    }
    void* dst = E->weights.take((size_t)(rows * cols) * es);
    put(dst, tmp.data(), rows * cols);
    return dst;
  };
  // decoder q/k/v rows head-major: row h * 192 + s * 64 + c = row h * 64 + c
  // of q_proj (s = 0), k_proj (1) or v_proj (2), so each head's rows are one
  // contiguous block (one thread-block cluster per head in the bf16 decode)
  auto head_qkv = [&](const std::string& p) {
    const float* w[3] = {fetch(p + "self_attn.q_proj.weight", in * d), fetch(p + "self_attn.k_proj.weight", in * d),
                         fetch(p + "self_attn.v_proj.weight", in * d)};
    tmp.resize((size_t)(3 * in * d));
    for (int64_t h = 0; h < c.num_heads; ++h)
      for (int sct = 0; sct < 3; ++sct)
        std::memcpy(&tmp[(size_t)((h * 192 + sct * 64) * d)], w[sct] + h * 64 * d, (size_t)(64 * d) * 4);
    void* dst = E->weights.take((size_t)(3 * in * d) * es);
    put(dst, tmp.data(), 3 * in * d);
    return dst;
  };
  // interleave wi_0 / wi_1 rows: row 2j = wi_0[j], row 2j+1 = wi_1[j]
  auto geglu = [&](const std::string& p) {
    const float* a = fetch(p + "ffn.wi_0.weight", ff * d);
    const float* b = fetch(p + "ffn.wi_1.weight", ff * d);
    tmp.resize((size_t)(2 * ff * d));
    for (int64_t j = 0; j < ff; ++j) {
      std::memcpy(&tmp[(size_t)((2 * j) * d)], a + j * d, (size_t)d * 4);
      std::memcpy(&tmp[(size_t)((2 * j + 1) * d)], b + j * d, (size_t)d * 4);
    }
    void* dst = E->weights.take((size_t)(2 * ff * d) * es);
    put(dst, tmp.data(), 2 * ff * d);
    return dst;
  };

  E->emb = single("token_embedding.weight", V * d);
  E->enc.resize(c.num_encoder_layers);
  for (int i = 0; i < c.num_encoder_layers; ++i) {
    const std::string p = "encoder_layers." + std::to_string(i) + ".";
    EncLayerDev& L = E->enc[i];
    L.wqkv = concat({{p + "self_attn.q_proj.weight", in}, {p + "self_attn.k_proj.weight", in},
                     {p + "self_attn.v_proj.weight", in}},
                    d);
    L.wo = single(p + "self_attn.o_proj.weight", d * in);
    L.n_attn = single(p + "pre_attn_norm.weight", d);
    L.wi = geglu(p);
    L.wout = single(p + "ffn.wo.weight", d * ff);
    L.n_ffn = single(p + "pre_ffn_norm.weight", d);
  }
  E->enc_norm = single("encoder_norm.weight", d);
  E->tl.resize(c.num_temporal_layers);
  for (int i = 0; i < c.num_temporal_layers; ++i) {
    const std::string p = "temporal_layers." + std::to_string(i) + ".";
    DecLayerDev& L = E->tl[i];
    L.wqkv = head_qkv(p);
    L.wo = single(p + "self_attn.o_proj.weight", d * in);
    L.n_self = single(p + "pre_self_attn_norm.weight", d);
    L.wcq = single(p + "cross_attn.q_proj.weight", in * d);
    L.wco = single(p + "cross_attn.o_proj.weight", d * in);
    L.n_cross = single(p + "pre_cross_attn_norm.weight", d);
    L.wi = geglu(p);
    L.wout = single(p + "ffn.wo.weight", d * ff);
    L.n_ffn = single(p + "pre_ffn_norm.weight", d);
  }
  {
    std::vector<std::pair<std::string, int64_t>> parts;
    for (int i = 0; i < c.num_temporal_layers; ++i) {
      const std::string p = "temporal_layers." + std::to_string(i) + ".";
      parts.push_back({p + "cross_attn.k_proj.weight", in});
      parts.push_back({p + "cross_attn.v_proj.weight", in});
    }
    E->wckv = concat(parts, d);
  }
  E->dl.resize(c.num_depth_layers);
  for (int i = 0; i < c.num_depth_layers; ++i) {
    const std::string p = "depth_layers." + std::to_string(i) + ".";
    DecLayerDev& L = E->dl[i];
    L.wqkv = head_qkv(p);
    L.wo = single(p + "self_attn.o_proj.weight", d * in);
    L.n_self = single(p + "pre_self_attn_norm.weight", d);
    L.wcq = L.wco = L.n_cross = nullptr;
    L.wi = geglu(p);
    L.wout = single(p + "ffn.wo.weight", d * ff);
    L.n_ffn = single(p + "pre_ffn_norm.weight", d);
  }
  E->dec_norm = single("decoder_norm.weight", d);
  E->lm_head = single("lm_head.weight", V * d);

  if (E->fused) {
    // o_proj (d, inner) -> [h][n][c]: row n = output dim, columns c < 64 =
    // head h's attention outputs, 8 zeros after (a CTA's block of output
    // dims is then one contiguous range, whatever the cluster size)
    const int64_t H = c.num_heads;
    auto o_block = [&](const std::string& key) {
      const float* w = fetch(key, d * in);
      tmp.assign((size_t)(H * d * 72), 0.f);
      for (int64_t h = 0; h < H; ++h)
        for (int64_t n = 0; n < d; ++n)
          for (int64_t cc = 0; cc < 64; ++cc) tmp[(size_t)(((h * d + n) * 72) + cc)] = w[n * in + h * 64 + cc];
      void* dst = E->weights.take(tmp.size() * es);
      put(dst, tmp.data(), (int64_t)tmp.size());
      return dst;
    };
    // wo (d, ff) -> [j][n][u]: row n = output dim, columns u < Uc = d_ff
    // units j * Uc + u of cluster j (zero past ff), 8 zeros after
    const int64_t NC = E->ffn_plan.nclusters, Uc = E->ffn_plan.Uc, Ur = Uc + 8;
    auto ffn_block = [&](const std::string& key) {
      const float* w = fetch(key, d * ff);
      tmp.assign((size_t)(NC * d * Ur), 0.f);
      for (int64_t j = 0; j < NC; ++j)
        for (int64_t n = 0; n < d; ++n)
          for (int64_t u = 0; u < Uc && j * Uc + u < ff; ++u)
            tmp[(size_t)(((j * d + n) * Ur) + u)] = w[n * ff + j * Uc + u];
      void* dst = E->weights.take(tmp.size() * es);
      put(dst, tmp.data(), (int64_t)tmp.size());
      return dst;
    };
    // a device copy of `rows` rows of `src` (compute dtype, d columns) with a
    // 16-byte zero pad after each row
    auto padded = [&](const void* src, int64_t rows) {
      const size_t rb = (size_t)d * es, rs = rb + 16;
      void* dst = E->weights.take((size_t)rows * rs);
      CUDA_OK(cudaMemset(dst, 0, (size_t)rows * rs));
      CUDA_OK(cudaMemcpy2D(dst, rs, src, rb, rb, (size_t)rows, cudaMemcpyDeviceToDevice));
      return dst;
    };
    for (int i = 0; i < c.num_temporal_layers; ++i) {
      DecLayerDev& L = E->tl[i];
      L.wqkv_pad = padded(L.wqkv, 3 * in);
      L.wcq_pad = padded(L.wcq, in);
      L.wi_pad = padded(L.wi, 2 * ff);
    }
    for (int i = 0; i < c.num_depth_layers; ++i) {
      DecLayerDev& L = E->dl[i];
      L.wqkv_pad = padded(L.wqkv, 3 * in);
      L.wi_pad = padded(L.wi, 2 * ff);
    }
    for (int i = 0; i < c.num_temporal_layers; ++i) {
      const std::string p = "temporal_layers." + std::to_string(i) + ".";
      E->tl[i].wo_blk = o_block(p + "self_attn.o_proj.weight");
      E->tl[i].wco_blk = o_block(p + "cross_attn.o_proj.weight");
      E->tl[i].wout_blk = ffn_block(p + "ffn.wo.weight");
    }
    for (int i = 0; i < c.num_depth_layers; ++i) {
      const std::string p = "depth_layers." + std::to_string(i) + ".";
      E->dl[i].wo_blk = o_block(p + "self_attn.o_proj.weight");
      E->dl[i].wout_blk = ffn_block(p + "ffn.wo.weight");
    }
  }

  // Relative-position bias per query position (precompute_*_biases,
  // model.cpp:302-320): bias[q][h][j] = table[bucket(j - q)][h], j <= q,
  // table values in the compute dtype (load_param casts, modules.cpp:127-128).
  auto bias_table = [&](const std::string& key, int nb, int maxd, int T) {
    const float* tab = fetch(key, (int64_t)nb * c.num_heads);
    std::vector<float> b((size_t)T * c.num_heads * T, 0.f);
    for (int q = 0; q < T; ++q)
      for (int j = 0; j <= q; ++j) {
        const int bk = relative_bucket(j - q, nb, maxd);
        for (int h = 0; h < c.num_heads; ++h) {
          float v = tab[(size_t)bk * c.num_heads + h];
          if (c.dtype == MRTDF_DTYPE_BF16) v = bf16_round_host(v);
          b[((size_t)q * c.num_heads + h) * T + j] = v;
        }
      }
    float* dst = (float*)E->weights.take(b.size() * 4);
    CUDA_OK(cudaMemcpy(dst, b.data(), b.size() * 4, cudaMemcpyHostToDevice));
    return dst;
  };
  E->tbias = bias_table("temporal_rel_pos.relative_attention_bias.weight", c.temporal_num_buckets,
                        c.temporal_max_distance, c.max_frames);
  E->dbias = bias_table("depth_rel_pos.relative_attention_bias.weight", c.depth_num_buckets, c.depth_max_distance,
                        c.rvq_depth);
  // Sinusoid table, cast to the compute dtype (model.cpp:232-235).
  std::vector<float> pe = sinusoid_table(c.max_encoder_length, (int)d);
  if (c.dtype == MRTDF_DTYPE_BF16)
    for (auto& v : pe) v = bf16_round_host(v);
  E->pe = (float*)E->weights.take(pe.size() * 4);
  CUDA_OK(cudaMemcpy(E->pe, pe.data(), pe.size() * 4, cudaMemcpyHostToDevice));
  E->loaded = true;
}

// ---------------------------------------------------------------------------
// Step sequences
// ---------------------------------------------------------------------------
namespace {

// A decode projection for more rows than the GEMV kernel takes (up to 128,
// bf16): RMSNorm rows (when the phase normalises) then the tcgen05 GEMM with
// the phase's epilogue; the batch rows are the MMA's M.
void wide_gemv(mrtdf_stream* st, int mode, bool norm, const GemvParams& p) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  const void* A = p.x;
  if (norm) {
    check_cuda(launch_rmsnorm_rows(c.dtype, p.x, p.norm_w, st->B, p.cols, st->xn, st->s, E->pdl), "rmsnorm");
    A = st->xn;
  }
  const int rpu = mode == kGemvGeglu ? 2 : 1;
  GemmParams g{};
  g.A = A; g.W = p.W; g.out = p.out; g.M = st->B; g.N = p.units * rpu; g.K = p.cols; g.lda = p.x_stride;
  g.ldo = p.out_stride;
  int epi = kEpiStore;
  switch (mode) {
    case kGemvStore: epi = kEpiStore; break;
    case kGemvResid: epi = kEpiDecResid; g.resid = p.resid; g.ldr = p.resid_stride; break;
    case kGemvGeglu: epi = kEpiGeglu; break;
    case kGemvLogits: epi = kEpiLogits; g.out_offset = p.out_offset; break;
    case kGemvQKV: epi = kEpiDecQKV; g.ck = p.kc; g.cv = p.vc; g.H = p.H; g.cap = p.cap; g.pos = p.pos; break;
    default: throw Error{MRTDF_ERR_INVALID, "wide decode path: unsupported projection"};
  }
  if (mode == kGemvStore && p.out_offset != 0) throw Error{MRTDF_ERR_INVALID, "wide decode path: column offset"};
  g.max_ksplit = E->wide_ksplit;
  check_cuda(launch_gemm_tc(epi, g, st->err, st->s, E->pdl), "wide decode gemm");
}

// In the measurement hook, whether the current stack's phases are enqueued.
// Key slices of the unfused cross attention: 8 for a few rows (latency), fewer
// once the (row, head) pairs alone fill the GPU several times over (64 CFG
// pairs: 2 slices, 503 -> 461 ms per chunk against 8; 1 or 4 slices are slower).
int cross_split(const mrtdf_stream* st) {
  const int pairs = st->B * st->eng->c.num_heads;
  if (pairs >= 512) return 2;
  if (pairs >= 256) return 4;
  return kCrossSplit;
}

bool phase_on(const mrtdf_stream* st) { return !st->gemv_only || (st->phase_mask & (st->in_depth ? 2 : 1)); }

void gemv(mrtdf_stream* st, int mode, bool norm, GemvParams p) {
  mrtdf_engine* E = st->eng;
  if (!phase_on(st)) return;
  p.err = st->err;
  p.B = st->B;
  // algorithmic bytes: weight rows + input rows + output rows (+ residual)
  const double es = E->esize;
  const int rpu = mode == kGemvGeglu ? 2 : 1;
  double bytes = (double)p.units * rpu * p.cols * es + (double)p.B * p.cols * es;
  bytes += (double)p.B * p.units * (mode == kGemvLogits ? 4.0 : es) * (mode == kGemvResid ? 2.0 : 1.0);
  if (norm) bytes += (double)p.cols * es;
  if (mode == kGemvQKVCluster)
    bytes += 2.0 * p.B * p.H * (p.pos + 1) * 64.0 * es;  // fused attention's K/V reads
  st->gemv_launches += 1;
  st->gemv_bytes += bytes;
  if (st->B > kGemvMaxB) {
    wide_gemv(st, mode, norm, p);
    return;
  }
  check_cuda(launch_gemv(E->c.dtype, mode, norm, p, E->num_sms, st->s, E->pdl), "gemv launch");
}

size_t act_bytes(const mrtdf_engine* E, size_t n) { return n * E->esize; }

// One DecoderLayer::forward for the stream's B rows at cache position
// `pos` (modules.cpp:384-408). x_in is read, the layer output lands in xr.
void enqueue_decoder_layer(mrtdf_stream* st, const DecLayerDev& L, const void* x_in, void* xr, void* kc, void* vc,
                           int cap, int pos, const float* bias, int bias_stride, const void* ck, const void* cv,
                           bool l2_keep) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  const int d = c.d_model, in = E->inner(), ff = c.d_ff;
  GemvParams p{};
  // 1. pre-norm + fused q/k/v, k/v appended to the cache at `pos`
  p.W = L.wqkv; p.x = x_in; p.norm_w = L.n_self; p.out = st->qb; p.kc = kc; p.vc = vc;
  p.units = 3 * in; p.cols = d; p.x_stride = d; p.out_stride = in; p.inner = in; p.H = c.num_heads;
  p.cap = cap; p.pos = pos; p.l2_keep = l2_keep;
  // 2. self attention with relative-position bias (scale 1.0): in bf16 fused
  // into the q/k/v kernel (the CTA completing a head attends it)
  if (E->cluster_attn && c.dtype == MRTDF_DTYPE_BF16 && st->B <= kQkvCluster) {
    p.bias = bias; p.bias_stride = bias_stride; p.attn_out = st->ao;
    gemv(st, kGemvQKVCluster, true, p);
  } else {
    gemv(st, kGemvQKV, true, p);
    AttnParams a{};
    a.q = st->qb; a.K = kc; a.V = vc; a.bias = bias; a.bias_stride = bias_stride; a.out = st->ao; a.err = st->err;
    a.B = st->B; a.H = c.num_heads; a.cap = cap; a.T = pos + 1; a.inner = in; a.nsplit = 1;
    if (!st->gemv_only) check_cuda(launch_attn_self(c.dtype, a, st->s, E->pdl), "attn_self launch");
  }
  // 3. o_proj + residual
  p = GemvParams{};
  p.W = L.wo; p.x = st->ao; p.out = xr; p.resid = x_in; p.units = d; p.cols = in; p.x_stride = in;
  p.out_stride = d; p.resid_stride = d; p.l2_keep = l2_keep;
  gemv(st, kGemvResid, false, p);
  if (ck) {
    // 4. pre-norm + cross q
    p = GemvParams{};
    p.W = L.wcq; p.x = xr; p.norm_w = L.n_cross; p.out = st->qb; p.units = in; p.cols = d; p.x_stride = d;
    p.out_stride = in; p.l2_keep = l2_keep;
    gemv(st, kGemvStore, true, p);
    // 5. cross attention over the cached encoder K/V
    AttnParams ca{};
    ca.q = st->qb; ca.K = ck; ca.V = cv; ca.bias = nullptr; ca.out = st->ao;
    ca.err = st->err; ca.B = st->B; ca.H = c.num_heads; ca.cap = c.max_encoder_length;
    ca.T = st->S; ca.inner = in; ca.nsplit = cross_split(st);
    if (!st->gemv_only) check_cuda(launch_attn_cross(c.dtype, ca, st->s, E->pdl), "attn_cross launch");
    // 6. cross o_proj + residual
    p = GemvParams{};
    p.W = L.wco; p.x = st->ao; p.out = xr; p.resid = xr; p.units = d; p.cols = in; p.x_stride = in;
    p.out_stride = d; p.resid_stride = d; p.l2_keep = l2_keep;
    gemv(st, kGemvResid, false, p);
  }
  // 7. pre-norm + wi_0 / wi_1 + gelu * gate
  p = GemvParams{};
  p.W = L.wi; p.x = xr; p.norm_w = L.n_ffn; p.out = st->hb; p.units = ff; p.cols = d; p.x_stride = d;
  p.out_stride = ff; p.l2_keep = l2_keep;
  gemv(st, kGemvGeglu, true, p);
  // 8. wo + residual
  p = GemvParams{};
  p.W = L.wout; p.x = st->hb; p.out = xr; p.resid = xr; p.units = d; p.cols = ff; p.x_stride = ff;
  p.out_stride = d; p.resid_stride = d; p.l2_keep = l2_keep;
  gemv(st, kGemvResid, false, p);
}

size_t layer_cache_elems(const mrtdf_stream* st, int cap) {
  return (size_t)st->B * st->eng->c.num_heads * cap * 64;
}

// ---- fused phases (bf16, at most two rows) ----------------------------------
// Start of a phase chain: the three accumulators are zero, the ring at 0.
void fused_reset(mrtdf_stream* st) {
  if (!st->fused) return;
  CUDA_OK(cudaMemsetAsync(st->facc, 0, (size_t)3 * st->B * st->eng->c.d_model * 8, st->s));
  st->fk = 0;
  st->fj = 0;
}

long long* facc_at(mrtdf_stream* st, int k) { return st->facc + (size_t)(k % 3) * st->B * st->eng->c.d_model; }

// Inputs / outputs of the next phase consuming `in`; returns the hidden
// state after that phase (its residual stream + the accumulator it adds to).
Hidden fused_io(mrtdf_stream* st, Hidden in, FusedIn& f) {
  if (in.acc && in.acc != facc_at(st, st->fk)) throw Error{MRTDF_ERR_STATE, "fused phase ring out of order"};
  f = FusedIn{};
  f.x = in.x;
  f.acc = in.acc;
  f.err = st->err;
  f.B = st->B;
  f.d = st->eng->c.d_model;
  const void* resid = in.x;
  if (in.acc) {
    f.x_out = st->fx[st->fj];
    resid = st->fx[st->fj];
    st->fj ^= 1;
  }
  f.acc_out = facc_at(st, st->fk + 1);
  f.acc_clear = facc_at(st, st->fk + 2);
  st->fk = (st->fk + 1) % 3;
  return Hidden{resid, f.acc_out};
}

// One DecoderLayer::forward as fused phases: self (+ cross) + FFN.
Hidden enqueue_fused_layer(mrtdf_stream* st, const DecLayerDev& L, Hidden in, void* kc, void* vc, int cap, int pos,
                           const float* bias, int bias_stride, const void* ck, const void* cv, bool l2_keep) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  const double es = E->esize, d = c.d_model, in_ = E->inner(), ff = c.d_ff, B = st->B;
  const bool on = phase_on(st);
  FusedSelfParams sp{};
  Hidden h = fused_io(st, in, sp.in);
  sp.wqkv = L.wqkv_pad; sp.norm_w = L.n_self; sp.wo_blk = L.wo_blk; sp.kc = kc; sp.vc = vc; sp.bias = bias;
  sp.bias_stride = bias_stride; sp.H = c.num_heads; sp.cap = cap; sp.pos = pos; sp.l2_keep = l2_keep;
  if (on) {
    check_cuda(launch_fused_self(sp, st->s, E->pdl), "fused self phase");
    st->gemv_launches += 1;
    st->gemv_bytes += (4.0 * in_ * d + d) * es + 2.0 * B * c.num_heads * (pos + 1) * 64.0 * es + 2.0 * B * d * es;
  }
  if (ck) {
    FusedCrossParams cp{};
    h = fused_io(st, h, cp.in);
    cp.wcq = L.wcq_pad; cp.norm_w = L.n_cross; cp.wco_blk = L.wco_blk; cp.ck = ck; cp.cv = cv; cp.H = c.num_heads;
    cp.Smax = c.max_encoder_length; cp.S = st->S; cp.l2_keep = l2_keep;
    if (on) {
      check_cuda(launch_fused_cross(cp, st->s, E->pdl), "fused cross phase");
      st->gemv_launches += 1;
      st->gemv_bytes += (2.0 * in_ * d + d) * es + 2.0 * B * c.num_heads * st->S * 64.0 * es + 2.0 * B * d * es;
    }
  }
  FusedFfnParams fp{};
  h = fused_io(st, h, fp.in);
  fp.wi = L.wi_pad; fp.norm_w = L.n_ffn; fp.wout_blk = L.wout_blk; fp.ff = c.d_ff; fp.Uc = E->ffn_plan.Uc;
  fp.nclusters = E->ffn_plan.nclusters; fp.l2_keep = l2_keep;
  if (on) {
    check_cuda(launch_fused_ffn(fp, st->s, E->pdl), "fused ffn phase");
    st->gemv_launches += 1;
    st->gemv_bytes += (3.0 * ff * d + d) * es + 2.0 * B * d * es;
  }
  return h;
}

// Write a hidden state out as plain bf16 rows (the step-level entry points).
void materialize(mrtdf_stream* st, Hidden h, void* out) {
  if (!h.acc) {
    if (h.x != out)
      CUDA_OK(cudaMemcpyAsync(out, h.x, act_bytes(st->eng, (size_t)st->B * st->eng->c.d_model),
                              cudaMemcpyDeviceToDevice, st->s));
    return;
  }
  FusedIn f{};
  f.x = h.x;
  f.acc = h.acc;
  f.B = st->B;
  f.d = st->eng->c.d_model;
  check_cuda(launch_fused_materialize(f, out, st->s, st->eng->pdl), "materialize");
}

// temporal_step: 20 decoder layers over tin (model.cpp:493-513). Returns
// the stack output (tx when the phases are not fused).
Hidden enqueue_temporal(mrtdf_stream* st, int f) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  const size_t tcs = layer_cache_elems(st, c.max_frames);
  const size_t ccs = layer_cache_elems(st, c.max_encoder_length);
  st->in_depth = false;
  Hidden h{st->tin, nullptr};
  for (int l = 0; l < c.num_temporal_layers; ++l) {
    uint8_t* tk = (uint8_t*)st->tk + act_bytes(E, tcs * l);
    uint8_t* tv = (uint8_t*)st->tv + act_bytes(E, tcs * l);
    const uint8_t* ck = (const uint8_t*)st->ck + act_bytes(E, ccs * l);
    const uint8_t* cv = (const uint8_t*)st->cv + act_bytes(E, ccs * l);
    const float* bias = E->tbias + (size_t)f * c.num_heads * c.max_frames;
    if (st->fused) {
      h = enqueue_fused_layer(st, E->tl[l], h, tk, tv, c.max_frames, f, bias, c.max_frames, ck, cv,
                              /*l2_keep=*/false);
    } else {
      enqueue_decoder_layer(st, E->tl[l], l == 0 ? st->tin : st->tx, st->tx, tk, tv, c.max_frames, f, bias,
                            c.max_frames, ck, cv, /*l2_keep=*/false);
      h = Hidden{st->tx, nullptr};
    }
  }
  return h;
}

// depth_step: 4 decoder layers + decoder_norm + lm_head rows [lo, hi).
void enqueue_depth(mrtdf_stream* st, int level, Hidden in, int lo, int hi) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  const size_t dcs = layer_cache_elems(st, c.rvq_depth);
  st->in_depth = true;
  Hidden h = in;
  for (int l = 0; l < c.num_depth_layers; ++l) {
    uint8_t* dk = (uint8_t*)st->dk + act_bytes(E, dcs * l);
    uint8_t* dv = (uint8_t*)st->dv + act_bytes(E, dcs * l);
    const float* bias = E->dbias + (size_t)level * c.num_heads * c.rvq_depth;
    if (st->fused) {
      h = enqueue_fused_layer(st, E->dl[l], h, dk, dv, c.rvq_depth, level, bias, c.rvq_depth, nullptr, nullptr,
                              /*l2_keep=*/true);
    } else {
      if (h.acc) throw Error{MRTDF_ERR_STATE, "depth_step: unfused layers need a plain input"};
      enqueue_decoder_layer(st, E->dl[l], l == 0 ? h.x : st->dx, st->dx, dk, dv, c.rvq_depth, level, bias,
                            c.rvq_depth, nullptr, nullptr, /*l2_keep=*/true);
    }
  }
  GemvParams p{};
  p.W = (const uint8_t*)E->lm_head + act_bytes(E, (size_t)lo * c.d_model);
  p.x = st->fused ? h.x : st->dx; p.acc = st->fused ? h.acc : nullptr;
  p.norm_w = E->dec_norm; p.out = st->logits; p.units = hi - lo; p.cols = c.d_model;
  p.x_stride = c.d_model; p.out_stride = c.vocab_size; p.out_offset = lo; p.l2_keep = 1;
  gemv(st, kGemvLogits, true, p);
  st->in_depth = false;
}

// encode: embed + PE, encoder layers, encoder_norm, cross K/V of every
// temporal layer (model.cpp:226-241, modules.cpp:323-333).
cudaError_t encoder_gemm(mrtdf_stream* st, int epi, const GemmParams& g) {
  mrtdf_engine* E = st->eng;
  if (E->c.dtype == MRTDF_DTYPE_BF16) return launch_gemm_tc(epi, g, st->err, st->s, E->pdl);
  return launch_gemm_f32(epi, g, st->s, E->pdl);
}

// One EncoderLayer (modules.cpp:349-358) over st->ex, (B * S, d), in place.
void enqueue_encoder_layer(mrtdf_stream* st, const EncLayerDev& L, int S) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  const int d = c.d_model, in = E->inner(), ff = c.d_ff;
  const int M = st->B * S;
  const int dt = c.dtype;
  const bool pdl = E->pdl;
  check_cuda(launch_rmsnorm_rows(dt, st->ex, L.n_attn, M, d, st->en, st->s, pdl), "rmsnorm");
  GemmParams g{};
  g.A = st->en; g.W = L.wqkv; g.out = st->eqkv; g.M = M; g.N = 3 * in; g.K = d; g.lda = d; g.ldo = 3 * in;
  check_cuda(encoder_gemm(st, kEpiStore, g), "gemm qkv");
  EncAttnParams a{st->eqkv, st->eo, st->B, S, c.num_heads, in, st->err};
  check_cuda(launch_enc_attention(dt, a, st->s, pdl), "enc attention");
  g = GemmParams{};
  g.A = st->eo; g.W = L.wo; g.out = st->ex; g.M = M; g.N = d; g.K = in; g.lda = in; g.ldo = d;
  check_cuda(encoder_gemm(st, kEpiResid, g), "gemm o");
  check_cuda(launch_rmsnorm_rows(dt, st->ex, L.n_ffn, M, d, st->en, st->s, pdl), "rmsnorm");
  g = GemmParams{};
  g.A = st->en; g.W = L.wi; g.out = st->eh; g.M = M; g.N = 2 * ff; g.K = d; g.lda = d; g.ldo = ff;
  check_cuda(encoder_gemm(st, kEpiGeglu, g), "gemm wi");
  g = GemmParams{};
  g.A = st->eh; g.W = L.wout; g.out = st->ex; g.M = M; g.N = d; g.K = ff; g.lda = ff; g.ldo = d;
  check_cuda(encoder_gemm(st, kEpiResid, g), "gemm wo");
}

void enqueue_encode(mrtdf_stream* st, int S) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  const int d = c.d_model, in = E->inner();
  const int M = st->B * S;
  const int dt = c.dtype;
  const bool pdl = E->pdl;
  check_cuda(launch_embed_pe(dt, E->emb, E->pe, st->ids, M, S, d, c.vocab_size, st->ex, st->err, st->s, pdl),
             "embed_pe");
  for (int l = 0; l < c.num_encoder_layers; ++l) enqueue_encoder_layer(st, E->enc[l], S);
  check_cuda(launch_rmsnorm_rows(dt, st->ex, E->enc_norm, M, d, st->en, st->s, pdl), "encoder_norm");
  GemmParams g{};
  g.A = st->en; g.W = E->wckv; g.out = nullptr; g.M = M; g.N = c.num_temporal_layers * 2 * in; g.K = d; g.lda = d;
  g.ck = st->ck; g.cv = st->cv; g.S = S; g.B = st->B; g.H = c.num_heads; g.Smax = c.max_encoder_length; g.inner = in;
  check_cuda(encoder_gemm(st, kEpiCrossKV, g), "gemm cross kv");
}

void enqueue_sample(mrtdf_stream* st, int f, int level, const mrtdf_gen_opts& o, bool masked, int lo, int hi,
                    bool forced) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  SampleParams sp{};
  sp.logits = st->logits; sp.logits_stride = c.vocab_size; sp.col_offset = 0; sp.lo = lo; sp.hi = hi;
  sp.rows_per_seq = st->rps; sp.w = o.guidance_weight; sp.temperature = o.temperature; sp.top_k = o.top_k;
  sp.seeds = st->seeds; sp.step = (uint32_t)(f * c.rvq_depth + level);
  sp.uniforms = o.uniforms ? st->uniforms + (size_t)sp.step * c.vocab_size : nullptr;
  sp.uni_seq_stride = (long long)o.num_frames * c.rvq_depth * c.vocab_size;
  sp.forced = forced ? st->forced : nullptr;
  sp.tokens = st->tokens; sp.tok_stride = c.max_frames * c.rvq_depth; sp.tok_index = f * c.rvq_depth + level;
  sp.emb = E->emb; sp.d = c.d_model; sp.V = c.vocab_size; sp.din = st->din; sp.fsum = st->fsum; sp.tin = st->tin;
  sp.depth = c.rvq_depth; sp.is_first = level == 0; sp.is_last = level == c.rvq_depth - 1; sp.err = st->err;
  sp.bad_token = 0;
  (void)masked;
  check_cuda(launch_sample(c.dtype, sp, st->nseq, st->s, E->pdl), "sample launch");
}

void level_range(const mrtdf_config& c, bool masked, int level, int& lo, int& hi) {
  if (masked) {
    lo = c.codec_offset + level * c.codebook_size;
    hi = lo + c.codebook_size;
  } else {
    lo = 0;
    hi = c.vocab_size;
  }
}

// The whole generate_tokens chunk (decode.cpp:364-513): PAD embedding for
// frame 0, temporal step, rvq_depth x (depth step + sampler).
void enqueue_chunk(mrtdf_stream* st, int S, const mrtdf_gen_opts& o) {
  mrtdf_engine* E = st->eng;
  const mrtdf_config& c = E->c;
  if (!st->gemv_only) {
    enqueue_encode(st, S);
    check_cuda(launch_embed_rows(c.dtype, E->emb, nullptr, st->B, c.d_model, st->tin, st->s, E->pdl), "embed pad");
  }
  const bool masked = o.use_vocab_masks != 0;
  fused_reset(st);
  for (int f = 0; f < o.num_frames; ++f) {
    const Hidden t = enqueue_temporal(st, f);
    for (int l = 0; l < c.rvq_depth; ++l) {
      int lo, hi;
      level_range(c, masked, l, lo, hi);
      enqueue_depth(st, l, l == 0 ? t : Hidden{st->din, nullptr}, lo, hi);
      if (!st->gemv_only) enqueue_sample(st, f, l, o, masked, lo, hi, false);
    }
  }
}

void validate_opts(const mrtdf_stream* st, const mrtdf_gen_opts* o, int seq_len) {
  const mrtdf_config& c = st->eng->c;
  if (!o) throw Error{MRTDF_ERR_INVALID, "opts is NULL"};
  if (o->num_frames <= 0 || o->num_frames > c.max_frames)
    throw Error{MRTDF_ERR_RANGE, "num_frames must be in [1, max_frames]"};
  if (o->rvq_depth != c.rvq_depth) throw Error{MRTDF_ERR_INVALID, "rvq_depth must equal the model's rvq_depth"};
  if (o->temperature < 0.f) throw Error{MRTDF_ERR_INVALID, "temperature must be >= 0"};
  if (seq_len <= 0 || seq_len > c.max_encoder_length)
    throw Error{MRTDF_ERR_RANGE, "seq_len exceeds max_encoder_length"};
  if (!o->use_vocab_masks && (size_t)c.vocab_size * 4 > 160 * 1024)
    throw Error{MRTDF_ERR_INVALID, "unmasked sampling supports vocab_size <= 40960"};
}

void upload_ids(mrtdf_stream* st, const int32_t* ids, int S) {
  const mrtdf_config& c = st->eng->c;
  for (size_t i = 0; i < (size_t)st->B * S; ++i)
    if (ids[i] < 0 || ids[i] >= c.vocab_size) throw Error{MRTDF_ERR_INVALID, "token id out of range"};
  CUDA_OK(cudaMemcpyAsync(st->ids, ids, (size_t)st->B * S * 4, cudaMemcpyHostToDevice, st->s));
}

void upload_seeds(mrtdf_stream* st, const mrtdf_gen_opts* o, const uint64_t* seeds) {
  std::vector<uint64_t> h(st->nseq);
  for (int i = 0; i < st->nseq; ++i) h[i] = seeds ? seeds[i] : o->seed + (uint64_t)i;
  CUDA_OK(cudaMemcpyAsync(st->seeds, h.data(), h.size() * 8, cudaMemcpyHostToDevice, st->s));
  CUDA_OK(cudaStreamSynchronize(st->s));  // h is a local
}

void upload_uniforms(mrtdf_stream* st, const mrtdf_gen_opts* o) {
  if (!o->uniforms) return;
  const mrtdf_config& c = st->eng->c;
  const size_t n = (size_t)st->nseq * o->num_frames * c.rvq_depth * c.vocab_size;
  if (n > st->uniforms_cap) {
    if (st->uniforms) cudaFree(st->uniforms);
    st->uniforms = nullptr;
    CUDA_OK(cudaMalloc(&st->uniforms, n * 4));
    st->uniforms_cap = n;
    for (auto& kv : st->graphs) cudaGraphExecDestroy(kv.second);
    st->graphs.clear();
  }
  CUDA_OK(cudaMemcpyAsync(st->uniforms, o->uniforms, n * 4, cudaMemcpyHostToDevice, st->s));
}

int read_err(mrtdf_stream* st) {
  int h = 0;
  CUDA_OK(cudaMemcpyAsync(&h, st->err, 4, cudaMemcpyDeviceToHost, st->s));
  CUDA_OK(cudaStreamSynchronize(st->s));
  if (h) {
    CUDA_OK(cudaMemsetAsync(st->err, 0, 4, st->s));
    CUDA_OK(cudaStreamSynchronize(st->s));
  }
  return h;
}

void check_device_err(mrtdf_stream* st) {
  const int h = read_err(st);
  if (h & (kErrMbarTimeout | kErrCounterTimeout))
    throw Error{MRTDF_ERR_TIMEOUT, "a device-side bounded wait gave up (error word " + std::to_string(h) + ")"};
  if (h & kErrFixedRange)
    throw Error{MRTDF_ERR_INVALID,
                "a decode activation left the range of the fixed-point split sums (NaN or |x| >= 2^30)"};
  if (h & kErrBadToken)
    throw Error{MRTDF_ERR_INVALID,
                "the sampler found no valid candidate (NaN logits or an empty vocabulary range) or an id outside the "
                "vocabulary"};
}

void run_chunk(mrtdf_stream* st, int S, const mrtdf_gen_opts& o) {
  GraphKey key{o.num_frames, o.rvq_depth, o.top_k, o.use_vocab_masks, o.uniforms != nullptr, S, o.temperature,
               o.guidance_weight};
  const bool use_graph = env_flag("MRTDF_GRAPH", true);
  if (!use_graph) {
    st->last_chunk_kernels = -1;  // counted only for graphs
    enqueue_chunk(st, S, o);
    return;
  }
  auto it = st->graphs.find(key);
  if (it == st->graphs.end()) {
    cudaGraph_t g = nullptr;
    CUDA_OK(cudaStreamBeginCapture(st->s, cudaStreamCaptureModeThreadLocal));
    try {
      enqueue_chunk(st, S, o);
    } catch (...) {
      cudaStreamEndCapture(st->s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    CUDA_OK(cudaStreamEndCapture(st->s, &g));
    size_t n = 0;
    long long kernels = 0;
    if (cudaGraphGetNodes(g, nullptr, &n) == cudaSuccess && n) {
      std::vector<cudaGraphNode_t> nodes(n);
      if (cudaGraphGetNodes(g, nodes.data(), &n) == cudaSuccess)
        for (size_t i = 0; i < n; ++i) {
          cudaGraphNodeType t;
          if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++kernels;
        }
    }
    cudaGraphExec_t ex = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    check_cuda(e, "cudaGraphInstantiate");
    it = st->graphs.emplace(key, ex).first;
    st->graph_kernels[key] = kernels;
  }
  st->last_chunk_kernels = st->graph_kernels[key];
  CUDA_OK(cudaGraphLaunch(it->second, st->s));
}

}  // namespace

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
extern "C" {

const char* mrtdf_last_error(void) { return last_error(); }

const char* mrtdf_version(void) { return "mrtdf 0.1.0 sm_100a"; }

int mrtdf_config_preset(const char* name, mrtdf_config* out) {
  return guarded([&] {
    if (!name || !out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (!config_preset(name, out)) throw Error{MRTDF_ERR_INVALID, std::string("unknown preset: ") + name};
  });
}

int mrtdf_write_random_safetensors(const mrtdf_config* cfg, uint64_t seed, float stddev, int norm_ones,
                                   const char* path) {
  return guarded([&] {
    if (!cfg || !path) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    const std::string why = config_check(*cfg);
    if (!why.empty()) throw Error{MRTDF_ERR_INVALID, why};
    auto hw = random_host_weights(*cfg, seed, stddev, norm_ones != 0);
    std::vector<OutTensor> ts;
    for (const auto& spec : weight_specs(*cfg)) ts.push_back({spec.key, spec.shape, hw->ptr.at(spec.key)});
    write_safetensors(path, ts);
  });
}

int mrtdf_create(const mrtdf_config* cfg, int device, mrtdf_engine** out) {
  return guarded([&] {
    if (!cfg || !out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    const std::string why = config_check(*cfg);
    if (!why.empty()) throw Error{MRTDF_ERR_INVALID, why};
    int n = 0;
    CUDA_OK(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n) throw Error{MRTDF_ERR_INVALID, "no such CUDA device"};
    CUDA_OK(cudaSetDevice(device));
    cudaDeviceProp prop;
    CUDA_OK(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10) throw Error{MRTDF_ERR_CUDA, std::string("built for sm_100a; device is ") + prop.name};
    auto E = std::make_unique<mrtdf_engine>();
    E->c = *cfg;
    E->device = device;
    E->num_sms = prop.multiProcessorCount;
    E->esize = cfg->dtype == MRTDF_DTYPE_BF16 ? 2 : 4;
    E->pdl = env_flag("MRTDF_PDL", true);
    E->cluster_attn = env_flag("MRTDF_CLUSTER_ATTN", true);
    if (const char* v = std::getenv("MRTDF_WIDE_KSPLIT")) E->wide_ksplit = std::max(1, std::min(8, std::atoi(v)));
    CUDA_OK(gemv_set_smem_limits());
    CUDA_OK(gemm_tc_set_smem_limits());
    CUDA_OK(fused_set_smem_limits());
    CUDA_OK(enc_attn_tc_set_smem_limits());
    E->fused = cfg->dtype == MRTDF_DTYPE_BF16 && env_flag("MRTDF_FUSED", true) &&
               fused_supported(cfg->d_model, cfg->num_heads, cfg->d_kv, cfg->d_ff);
    if (E->fused && fused_ffn_plan(cfg->d_model, cfg->d_ff, E->num_sms, &E->ffn_plan) != cudaSuccess) {
      cudaGetLastError();  // no FFN plan fits this device: the per-projection path serves every stream
      E->fused = false;
    }
    CUDA_OK(sample_set_smem_limits());
    *out = E.release();
  });
}

int mrtdf_destroy(mrtdf_engine* eng) {
  return guarded([&] {
    if (!eng) return;
    cudaSetDevice(eng->device);
    delete eng;
  });
}

int mrtdf_load_safetensors(mrtdf_engine* E, const char* path) {
  return guarded([&] {
    if (!E || !path) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    CUDA_OK(cudaSetDevice(E->device));
    SafetensorsFile f(path);
    std::map<std::string, std::vector<float>> conv;
    WeightSource src;
    src.get = [&](const std::string& key, int64_t n) -> const float* {
      const TensorRef* t = f.find(key);
      if (!t) throw Error{MRTDF_ERR_KEY, "WeightBundle " + std::string(path) + ": missing key \"" + key + "\""};
      if (t->numel() != n) throw Error{MRTDF_ERR_INVALID, "shape mismatch for " + key};
      if (t->dtype == "F32") return reinterpret_cast<const float*>(t->data);
      auto& v = conv[key];
      v.resize((size_t)n);
      const uint16_t* s = reinterpret_cast<const uint16_t*>(t->data);
      for (int64_t i = 0; i < n; ++i) {
        const uint32_t u = (uint32_t)s[i] << 16;
        std::memcpy(&v[(size_t)i], &u, 4);
      }
      return v.data();
    };
    upload_weights(E, src);
  });
}

int mrtdf_load_random(mrtdf_engine* E, uint64_t seed, float stddev, int norm_ones) {
  return guarded([&] {
    if (!E) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    CUDA_OK(cudaSetDevice(E->device));
    auto hw = random_host_weights(E->c, seed, stddev, norm_ones != 0);
    WeightSource src;
    src.get = [&](const std::string& key, int64_t n) -> const float* {
      auto it = hw->ptr.find(key);
      if (it == hw->ptr.end()) throw Error{MRTDF_ERR_KEY, "missing key \"" + key + "\""};
      (void)n;
      return it->second;
    };
    upload_weights(E, src);
  });
}

int mrtdf_stream_create(mrtdf_engine* E, int num_sequences, int cfg, mrtdf_stream** out) {
  return guarded([&] {
    if (!E || !out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (!E->loaded) throw Error{MRTDF_ERR_STATE, "load weights before creating a stream"};
    if (num_sequences <= 0) throw Error{MRTDF_ERR_INVALID, "num_sequences must be positive"};
    const int rps = cfg ? 2 : 1;
    const int max_rows = E->c.dtype == MRTDF_DTYPE_BF16 ? kWideMaxRows : kGemvMaxB;
    if (num_sequences * rps > max_rows)
      throw Error{MRTDF_ERR_INVALID, "rows per step (num_sequences * (cfg ? 2 : 1)) must be <= " +
                                         std::to_string(max_rows) + " (8 in fp32, 128 in bf16)"};
    CUDA_OK(cudaSetDevice(E->device));
    const mrtdf_config& c = E->c;
    auto st = std::make_unique<mrtdf_stream>();
    st->eng = E;
    st->nseq = num_sequences;
    st->rps = rps;
    st->B = num_sequences * rps;
    CUDA_OK(cudaStreamCreateWithFlags(&st->s, cudaStreamNonBlocking));
    const size_t B = st->B, d = c.d_model, in = E->inner(), ff = c.d_ff, V = c.vocab_size, H = c.num_heads;
    const size_t es = E->esize;
    const size_t Mx = B * c.max_encoder_length;
    std::vector<std::pair<void**, size_t>> plan = {
        {&st->tx, B * d * es}, {&st->dx, B * d * es}, {&st->tin, B * d * es}, {&st->din, B * d * es},
        {&st->fsum, B * d * es}, {&st->qb, B * in * es}, {&st->ao, B * in * es}, {&st->hb, B * ff * 4},
        {(void**)&st->logits, B * V * 4}, {(void**)&st->stage_f32, B * std::max(d, V) * 4},
        {&st->tk, c.num_temporal_layers * B * H * c.max_frames * 64 * es},
        {&st->tv, c.num_temporal_layers * B * H * c.max_frames * 64 * es},
        {&st->ck, c.num_temporal_layers * B * H * c.max_encoder_length * 64 * es},
        {&st->cv, c.num_temporal_layers * B * H * c.max_encoder_length * 64 * es},
        {&st->dk, c.num_depth_layers * B * H * c.rvq_depth * 64 * es},
        {&st->dv, c.num_depth_layers * B * H * c.rvq_depth * 64 * es},
        {&st->ex, Mx * d * es}, {&st->en, Mx * d * es}, {&st->eqkv, Mx * 3 * in * es}, {&st->eo, Mx * in * es},
        {&st->eh, Mx * ff * es}, {(void**)&st->ids, Mx * 4}, {&st->xn, B * d * es},
        {(void**)&st->tokens, (size_t)num_sequences * c.max_frames * c.rvq_depth * 4},
        {(void**)&st->seeds, (size_t)num_sequences * 8}, {(void**)&st->forced, (size_t)num_sequences * 4},
        {(void**)&st->err, 64}};
    st->fused = E->fused && st->B <= kFusedMaxRows;
    if (st->fused) {
      plan.push_back({(void**)&st->facc, 3 * B * d * 8});
      plan.push_back({&st->fx[0], B * d * es});
      plan.push_back({&st->fx[1], B * d * es});
    }
    size_t total = 0;
    for (auto& p : plan) total += (p.second + 255) & ~(size_t)255;
    st->mem.reserve(total);
    for (auto& p : plan) *p.first = st->mem.take(p.second);
    CUDA_OK(cudaMemsetAsync(st->mem.base, 0, st->mem.cap, st->s));
    CUDA_OK(cudaStreamSynchronize(st->s));
    *out = st.release();
  });
}

int mrtdf_stream_destroy(mrtdf_stream* st) {
  return guarded([&] {
    if (!st) return;
    cudaSetDevice(st->eng->device);
    cudaStreamSynchronize(st->s);
    if (st->uniforms) cudaFree(st->uniforms);
    if (st->seed_table) cudaFree(st->seed_table);
    delete st;
  });
}

int mrtdf_stream_rows(const mrtdf_stream* st) { return st ? st->B : 0; }

void* mrtdf_stream_cuda(mrtdf_stream* st) { return st ? (void*)st->s : nullptr; }

int mrtdf_check_wait_timeout(mrtdf_stream* st, int timeout_us) {
  return guarded([&] {
    if (!st) throw Error{MRTDF_ERR_INVALID, "NULL stream"};
    if (timeout_us < 1 || timeout_us > 1000000) throw Error{MRTDF_ERR_RANGE, "timeout_us must be in [1, 1e6]"};
    CUDA_OK(cudaSetDevice(st->eng->device));
    check_cuda(launch_wait_timeout_probe(st->err, (unsigned long long)timeout_us * 1000ull, st->s), "probe launch");
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
  });
}

int mrtdf_stream_sync(mrtdf_stream* st) {
  return guarded([&] {
    if (!st) throw Error{MRTDF_ERR_INVALID, "NULL stream"};
    CUDA_OK(cudaSetDevice(st->eng->device));
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
  });
}

int mrtdf_encode(mrtdf_stream* st, const int32_t* ids, int seq_len, float* enc_out) {
  return guarded([&] {
    if (!st || !ids) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    mrtdf_engine* E = st->eng;
    if (seq_len <= 0 || seq_len > E->c.max_encoder_length)
      throw Error{MRTDF_ERR_RANGE, "seq_len exceeds max_encoder_length"};
    CUDA_OK(cudaSetDevice(E->device));
    upload_ids(st, ids, seq_len);
    enqueue_encode(st, seq_len);
    st->S = seq_len;
    st->encoded = true;
    st->t_len = 0;
    st->d_len = 0;
    st->have_temporal = false;
    if (enc_out) {
      const size_t n = (size_t)st->B * seq_len * E->c.d_model;
      float* tmp = nullptr;
      CUDA_OK(cudaMalloc(&tmp, n * 4));
      check_cuda(launch_act_to_f32(E->c.dtype, st->en, n, tmp, st->s), "convert");
      CUDA_OK(cudaMemcpyAsync(enc_out, tmp, n * 4, cudaMemcpyDeviceToHost, st->s));
      CUDA_OK(cudaStreamSynchronize(st->s));
      cudaFree(tmp);
    }
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
  });
}

static void upload_act(mrtdf_stream* st, const float* x, void* dst) {
  mrtdf_engine* E = st->eng;
  const size_t n = (size_t)st->B * E->c.d_model;
  CUDA_OK(cudaMemcpyAsync(st->stage_f32, x, n * 4, cudaMemcpyHostToDevice, st->s));
  check_cuda(launch_f32_to_act(E->c.dtype, st->stage_f32, n, dst, st->s), "convert");
}

static void download_act(mrtdf_stream* st, const void* src, float* out) {
  mrtdf_engine* E = st->eng;
  const size_t n = (size_t)st->B * E->c.d_model;
  check_cuda(launch_act_to_f32(E->c.dtype, src, n, st->stage_f32, st->s), "convert");
  CUDA_OK(cudaMemcpyAsync(out, st->stage_f32, n * 4, cudaMemcpyDeviceToHost, st->s));
}

int mrtdf_temporal_step(mrtdf_stream* st, const float* x, int frame_idx, float* out) {
  return guarded([&] {
    if (!st) throw Error{MRTDF_ERR_INVALID, "NULL stream"};
    mrtdf_engine* E = st->eng;
    if (!st->encoded) throw Error{MRTDF_ERR_STATE, "temporal_step: call encode first (no cross-attention cache)"};
    if (frame_idx < 0 || frame_idx >= E->c.max_frames) throw Error{MRTDF_ERR_RANGE, "frame_idx out of range"};
    if (frame_idx != st->t_len) throw Error{MRTDF_ERR_STATE, "temporal_step: cache size mismatch"};
    CUDA_OK(cudaSetDevice(E->device));
    if (x) upload_act(st, x, st->tin);
    else check_cuda(launch_embed_rows(E->c.dtype, E->emb, nullptr, st->B, E->c.d_model, st->tin, st->s, false), "pad");
    fused_reset(st);
    materialize(st, enqueue_temporal(st, frame_idx), st->tx);
    st->t_len = frame_idx + 1;
    st->have_temporal = true;
    if (out) download_act(st, st->tx, out);
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
  });
}

int mrtdf_depth_step(mrtdf_stream* st, const float* x, int depth_idx, float* logits) {
  return guarded([&] {
    if (!st) throw Error{MRTDF_ERR_INVALID, "NULL stream"};
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    if (depth_idx < 0 || depth_idx >= c.rvq_depth) throw Error{MRTDF_ERR_RANGE, "depth_idx out of range"};
    if (depth_idx != 0 && depth_idx != st->d_len) throw Error{MRTDF_ERR_STATE, "depth_step: cache size mismatch"};
    CUDA_OK(cudaSetDevice(E->device));
    const void* in;
    if (x) {
      upload_act(st, x, st->din);
      in = st->din;
    } else {
      if (!st->have_temporal) throw Error{MRTDF_ERR_STATE, "depth_step: no temporal output to start from"};
      in = st->tx;
    }
    fused_reset(st);
    enqueue_depth(st, depth_idx, Hidden{in, nullptr}, 0, c.vocab_size);
    st->d_len = depth_idx + 1;
    if (logits)
      CUDA_OK(cudaMemcpyAsync(logits, st->logits, (size_t)st->B * c.vocab_size * 4, cudaMemcpyDeviceToHost, st->s));
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
  });
}

int mrtdf_token_embedding(mrtdf_engine* E, const int32_t* ids, int n, float* out) {
  return guarded([&] {
    if (!E || !ids || !out || n <= 0) throw Error{MRTDF_ERR_INVALID, "bad argument"};
    if (!E->loaded) throw Error{MRTDF_ERR_STATE, "weights not loaded"};
    for (int i = 0; i < n; ++i)
      if (ids[i] < 0 || ids[i] >= E->c.vocab_size) throw Error{MRTDF_ERR_INVALID, "token id out of range"};
    CUDA_OK(cudaSetDevice(E->device));
    const size_t dn = (size_t)n * E->c.d_model;
    int32_t* dids = nullptr;
    void* act = nullptr;
    float* f = nullptr;
    CUDA_OK(cudaMalloc(&dids, (size_t)n * 4));
    CUDA_OK(cudaMalloc(&act, dn * E->esize));
    CUDA_OK(cudaMalloc(&f, dn * 4));
    CUDA_OK(cudaMemcpy(dids, ids, (size_t)n * 4, cudaMemcpyHostToDevice));
    check_cuda(launch_embed_rows(E->c.dtype, E->emb, dids, n, E->c.d_model, act, 0, false), "embed");
    check_cuda(launch_act_to_f32(E->c.dtype, act, dn, f, 0), "convert");
    CUDA_OK(cudaMemcpy(out, f, dn * 4, cudaMemcpyDeviceToHost));
    cudaFree(dids);
    cudaFree(act);
    cudaFree(f);
  });
}

int mrtdf_sample(mrtdf_engine* E, const float* logits, int cfg, int frame, int level, const mrtdf_gen_opts* o,
                 const float* uniforms, int32_t* token) {
  return guarded([&] {
    if (!E || !logits || !o || !token) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (!E->loaded) throw Error{MRTDF_ERR_STATE, "weights not loaded"};
    const mrtdf_config& c = E->c;
    if (level < 0 || level >= c.rvq_depth || frame < 0) throw Error{MRTDF_ERR_RANGE, "level / frame out of range"};
    if (!o->use_vocab_masks && (size_t)c.vocab_size * 4 > 160 * 1024)
      throw Error{MRTDF_ERR_INVALID, "unmasked sampling supports vocab_size <= 40960"};
    CUDA_OK(cudaSetDevice(E->device));
    const int rows = cfg ? 2 : 1;
    const size_t V = c.vocab_size, d = c.d_model;
    float *dl = nullptr, *du = nullptr;
    int32_t* dt = nullptr;
    void *din = nullptr, *fs = nullptr, *tin = nullptr;
    int* err = nullptr;
    CUDA_OK(cudaMalloc(&dl, rows * V * 4));
    CUDA_OK(cudaMalloc(&dt, 4));
    CUDA_OK(cudaMalloc(&din, rows * d * E->esize));
    CUDA_OK(cudaMalloc(&fs, rows * d * E->esize));
    CUDA_OK(cudaMalloc(&tin, rows * d * E->esize));
    CUDA_OK(cudaMalloc(&err, 4));
    CUDA_OK(cudaMemset(err, 0, 4));
    CUDA_OK(cudaMemcpy(dl, logits, rows * V * 4, cudaMemcpyHostToDevice));
    if (uniforms) {
      CUDA_OK(cudaMalloc(&du, V * 4));
      CUDA_OK(cudaMemcpy(du, uniforms, V * 4, cudaMemcpyHostToDevice));
    }
    int lo, hi;
    level_range(c, o->use_vocab_masks != 0, level, lo, hi);
    SampleParams sp{};
    sp.logits = dl; sp.logits_stride = (int)V; sp.col_offset = 0; sp.lo = lo; sp.hi = hi; sp.rows_per_seq = rows;
    sp.w = o->guidance_weight; sp.temperature = o->temperature; sp.top_k = o->top_k; sp.seeds = nullptr;
    sp.seed_value = o->seed;
    sp.step = (uint32_t)(frame * c.rvq_depth + level);
    sp.uniforms = du;  // one row of V draws for this step
    sp.uni_seq_stride = 0; sp.forced = nullptr; sp.tokens = dt; sp.tok_stride = 0; sp.tok_index = 0;
    sp.emb = E->emb; sp.d = (int)d; sp.V = (int)V; sp.din = din; sp.fsum = fs; sp.tin = tin; sp.depth = c.rvq_depth;
    sp.is_first = 1; sp.is_last = 0; sp.err = err; sp.bad_token = -1;
    check_cuda(launch_sample(c.dtype, sp, 1, 0, false), "sample");
    int herr = 0;
    CUDA_OK(cudaMemcpy(token, dt, 4, cudaMemcpyDeviceToHost));
    CUDA_OK(cudaMemcpy(&herr, err, 4, cudaMemcpyDeviceToHost));
    cudaFree(dl); cudaFree(dt); cudaFree(din); cudaFree(fs); cudaFree(tin); cudaFree(err);
    if (du) cudaFree(du);
    if (herr & kErrBadToken)
      throw Error{MRTDF_ERR_INVALID, "sample: no candidate could be drawn (NaN logits or an empty vocabulary range)"};
  });
}

int mrtdf_sample_noalloc(mrtdf_engine* E, const float* logits_dev, int cfg, int frame, int level,
                         const mrtdf_gen_opts* o, const float* uniforms_dev, int32_t* token_dev, void* stream) {
  return guarded([&] {
    if (!E || !logits_dev || !o || !token_dev) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (!E->loaded) throw Error{MRTDF_ERR_STATE, "weights not loaded"};
    const mrtdf_config& c = E->c;
    if (level < 0 || level >= c.rvq_depth || frame < 0) throw Error{MRTDF_ERR_RANGE, "level / frame out of range"};
    if (!o->use_vocab_masks && (size_t)c.vocab_size * 4 > kSampleMaxSmem)
      throw Error{MRTDF_ERR_INVALID, "unmasked sampling supports vocab_size <= 40960"};
    const int rows = cfg ? 2 : 1;
    const size_t row_bytes = (size_t)rows * c.d_model * E->esize;
    if (row_bytes > kSampleScratchRowBytes)
      throw Error{MRTDF_ERR_RANGE, "mrtdf_sample_noalloc: rows x d_model x dtype bytes = " + std::to_string(row_bytes) +
                                       " exceeds its fixed scratch of " + std::to_string(kSampleScratchRowBytes) +
                                       " bytes per feedback row"};
    CUDA_OK(cudaSetDevice(E->device));
    void* scratch = nullptr;
    CUDA_OK(sample_scratch_address(E->device, &scratch));
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    uint8_t* base = reinterpret_cast<uint8_t*>(scratch);
    int lo, hi;
    level_range(c, o->use_vocab_masks != 0, level, lo, hi);
    SampleParams sp{};
    sp.logits = logits_dev; sp.logits_stride = c.vocab_size; sp.col_offset = 0; sp.lo = lo; sp.hi = hi;
    sp.rows_per_seq = rows; sp.w = o->guidance_weight; sp.temperature = o->temperature; sp.top_k = o->top_k;
    sp.seeds = nullptr; sp.seed_value = o->seed; sp.step = (uint32_t)(frame * c.rvq_depth + level);
    sp.uniforms = uniforms_dev; sp.uni_seq_stride = 0; sp.forced = nullptr;
    sp.tokens = token_dev; sp.tok_stride = 0; sp.tok_index = 0;
    sp.emb = E->emb; sp.d = c.d_model; sp.V = c.vocab_size;
    sp.din = base + 256;
    sp.fsum = base + 256 + kSampleScratchRowBytes;
    sp.tin = base + 256 + 2 * kSampleScratchRowBytes;
    // no error word: a failed draw stores -1 as the token
    sp.depth = c.rvq_depth; sp.is_first = 1; sp.is_last = 0; sp.err = nullptr; sp.bad_token = -1;
    check_cuda(launch_sample(c.dtype, sp, 1, s, false), "sample launch");
  });
}

int mrtdf_generate_tokens_dev(mrtdf_stream* st, const int32_t* enc_ids_dev, int seq_len, const mrtdf_gen_opts* o,
                              const uint64_t* seeds, int32_t* out_ids_dev) {
  return guarded([&] {
    if (!st || !enc_ids_dev || !out_ids_dev) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    validate_opts(st, o, seq_len);
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    CUDA_OK(cudaSetDevice(E->device));
    CUDA_OK(cudaMemcpyAsync(st->ids, enc_ids_dev, (size_t)st->B * seq_len * 4, cudaMemcpyDeviceToDevice, st->s));
    upload_seeds(st, o, seeds);
    upload_uniforms(st, o);
    st->S = seq_len;
    run_chunk(st, seq_len, *o);
    // tokens (nseq, max_frames, depth) -> out (nseq, num_frames, depth)
    CUDA_OK(cudaMemcpy2DAsync(out_ids_dev, (size_t)o->num_frames * c.rvq_depth * 4, st->tokens,
                              (size_t)c.max_frames * c.rvq_depth * 4, (size_t)o->num_frames * c.rvq_depth * 4,
                              st->nseq, cudaMemcpyDeviceToDevice, st->s));
    st->encoded = true;
    st->t_len = o->num_frames;
    st->d_len = c.rvq_depth;
    st->have_temporal = true;
  });
}

int mrtdf_generate_stream_dev(mrtdf_stream* st, int32_t* context_dev, int ctx_frames, int enc_depth,
                              const int32_t* style_dev, int style_depth, int num_chunks, const mrtdf_gen_opts* o,
                              const uint64_t* seeds, int32_t* rvq_out_dev) {
  return guarded([&] {
    if (!st || !context_dev || !o || !rvq_out_dev || (style_depth > 0 && !style_dev))
      throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    if (ctx_frames <= 0 || enc_depth <= 0 || enc_depth > c.rvq_depth || style_depth < 0 || num_chunks <= 0)
      throw Error{MRTDF_ERR_INVALID, "bad sizes"};
    const int S = ctx_frames * enc_depth + style_depth;
    validate_opts(st, o, S);
    if (o->uniforms) throw Error{MRTDF_ERR_INVALID, "streaming draws with Philox (no injected uniforms)"};
    if (o->num_frames > ctx_frames) throw Error{MRTDF_ERR_INVALID, "a chunk is longer than the context"};
    GlueParams gp{};
    gp.context = context_dev; gp.style = style_dev; gp.ids = st->ids; gp.tokens = st->tokens; gp.err = st->err;
    gp.nseq = st->nseq; gp.rows_per_seq = st->rps; gp.ctx_frames = ctx_frames; gp.rvq_depth = c.rvq_depth;
    gp.enc_depth = enc_depth; gp.style_depth = style_depth; gp.frames = o->num_frames;
    gp.tok_stride = c.max_frames * c.rvq_depth; gp.codebook_size = c.codebook_size; gp.codec_offset = c.codec_offset;
    if (glue_roll_smem(gp) > kGlueMaxSmem) throw Error{MRTDF_ERR_RANGE, "context too long for the device roll"};
    CUDA_OK(cudaSetDevice(E->device));
    // seeds of every chunk: seeds[chunk * nseq + i], or opts->seed + chunk for
    // sequence 0 (the CLI's seed + chunk_index) and + i << 32 for sequence i
    const size_t n = (size_t)num_chunks * st->nseq;
    std::vector<uint64_t> h(n);
    for (int k = 0; k < num_chunks; ++k)
      for (int i = 0; i < st->nseq; ++i)
        h[(size_t)k * st->nseq + i] = seeds ? seeds[(size_t)k * st->nseq + i] : o->seed + k + ((uint64_t)i << 32);
    if (n > st->seed_table_cap) {
      CUDA_OK(cudaStreamSynchronize(st->s));
      if (st->seed_table) cudaFree(st->seed_table);
      st->seed_table = nullptr;
      CUDA_OK(cudaMalloc(&st->seed_table, n * 8));
      st->seed_table_cap = n;
    }
    CUDA_OK(cudaMemcpyAsync(st->seed_table, h.data(), n * 8, cudaMemcpyHostToDevice, st->s));
    CUDA_OK(cudaStreamSynchronize(st->s));  // h is a local
    st->S = S;
    for (int k = 0; k < num_chunks; ++k) {
      CUDA_OK(cudaMemcpyAsync(st->seeds, st->seed_table + (size_t)k * st->nseq, (size_t)st->nseq * 8,
                              cudaMemcpyDeviceToDevice, st->s));
      check_cuda(launch_stream_encoder_ids(gp, st->s), "encoder ids");
      run_chunk(st, S, *o);
      gp.rvq_out = rvq_out_dev + (size_t)k * st->nseq * o->num_frames * c.rvq_depth;
      check_cuda(launch_stream_roll(gp, st->s), "context roll");
    }
    st->encoded = true;
    st->t_len = o->num_frames;
    st->d_len = c.rvq_depth;
    st->have_temporal = true;
  });
}

int mrtdf_generate_tokens(mrtdf_stream* st, const int32_t* enc_ids, int seq_len, const mrtdf_gen_opts* o,
                          const uint64_t* seeds, int32_t* out_ids) {
  return guarded([&] {
    if (!st || !enc_ids || !out_ids) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    validate_opts(st, o, seq_len);
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    CUDA_OK(cudaSetDevice(E->device));
    upload_ids(st, enc_ids, seq_len);
    upload_seeds(st, o, seeds);
    upload_uniforms(st, o);
    st->S = seq_len;
    run_chunk(st, seq_len, *o);
    CUDA_OK(cudaMemcpy2DAsync(out_ids, (size_t)o->num_frames * c.rvq_depth * 4, st->tokens,
                              (size_t)c.max_frames * c.rvq_depth * 4, (size_t)o->num_frames * c.rvq_depth * 4,
                              st->nseq, cudaMemcpyDeviceToHost, st->s));
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
    st->encoded = true;
    st->t_len = o->num_frames;
    st->d_len = c.rvq_depth;
    st->have_temporal = true;
  });
}

int mrtdf_teacher_forced_logits(mrtdf_stream* st, const int32_t* enc_ids, int seq_len, const int32_t* tokens,
                                int num_frames, float* logits) {
  return guarded([&] {
    if (!st || !enc_ids || !tokens || !logits) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    if (st->nseq != 1) throw Error{MRTDF_ERR_INVALID, "teacher forcing needs a single-sequence stream"};
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    if (num_frames <= 0 || num_frames > c.max_frames) throw Error{MRTDF_ERR_RANGE, "num_frames out of range"};
    if (seq_len <= 0 || seq_len > c.max_encoder_length) throw Error{MRTDF_ERR_RANGE, "seq_len out of range"};
    for (int i = 0; i < num_frames * c.rvq_depth; ++i)
      if (tokens[i] < 0 || tokens[i] >= c.vocab_size) throw Error{MRTDF_ERR_INVALID, "forced token out of range"};
    CUDA_OK(cudaSetDevice(E->device));
    upload_ids(st, enc_ids, seq_len);
    st->S = seq_len;
    mrtdf_gen_opts o{};
    o.num_frames = num_frames;
    o.rvq_depth = c.rvq_depth;
    upload_seeds(st, &o, nullptr);
    enqueue_encode(st, seq_len);
    check_cuda(launch_embed_rows(c.dtype, E->emb, nullptr, st->B, c.d_model, st->tin, st->s, false), "pad");
    const size_t V = c.vocab_size;
    fused_reset(st);
    for (int f = 0; f < num_frames; ++f) {
      const Hidden t = enqueue_temporal(st, f);
      for (int l = 0; l < c.rvq_depth; ++l) {
        enqueue_depth(st, l, l == 0 ? t : Hidden{st->din, nullptr}, 0, c.vocab_size);
        CUDA_OK(cudaMemcpyAsync(logits + ((size_t)f * c.rvq_depth + l) * st->B * V, st->logits,
                                (size_t)st->B * V * 4, cudaMemcpyDeviceToHost, st->s));
        const int32_t tok = tokens[(size_t)f * c.rvq_depth + l];
        CUDA_OK(cudaMemcpyAsync(st->forced, &tok, 4, cudaMemcpyHostToDevice, st->s));
        enqueue_sample(st, f, l, o, false, 0, c.vocab_size, true);
        CUDA_OK(cudaStreamSynchronize(st->s));  // `tok` is a local
      }
    }
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
    st->encoded = true;
    st->t_len = num_frames;
    st->d_len = c.rvq_depth;
    st->have_temporal = true;
  });
}

int mrtdf_bench_phases(mrtdf_stream* st, const mrtdf_gen_opts* o, int stack_mask, int reps, float* ms_per_rep,
                       long long* launches_per_rep, double* bytes_per_rep) {
  return guarded([&] {
    if (!st || !o || reps <= 0 || !ms_per_rep || !launches_per_rep || !bytes_per_rep || stack_mask < 1 || stack_mask > 3)
      throw Error{MRTDF_ERR_INVALID, "bad argument"};
    if (!st->encoded) throw Error{MRTDF_ERR_STATE, "run a chunk (or encode) first"};
    validate_opts(st, o, st->S);
    CUDA_OK(cudaSetDevice(st->eng->device));
    cudaGraph_t g = nullptr;
    st->gemv_only = true;
    st->phase_mask = stack_mask;
    st->gemv_launches = 0;
    st->gemv_bytes = 0.0;
    CUDA_OK(cudaStreamBeginCapture(st->s, cudaStreamCaptureModeThreadLocal));
    try {
      enqueue_chunk(st, st->S, *o);
    } catch (...) {
      st->gemv_only = false;
      st->phase_mask = 3;
      cudaStreamEndCapture(st->s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    st->gemv_only = false;
    st->phase_mask = 3;
    CUDA_OK(cudaStreamEndCapture(st->s, &g));
    cudaGraphExec_t ex = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    check_cuda(e, "cudaGraphInstantiate");
    cudaEvent_t a, b;
    CUDA_OK(cudaEventCreate(&a));
    CUDA_OK(cudaEventCreate(&b));
    CUDA_OK(cudaGraphLaunch(ex, st->s));  // warm-up
    CUDA_OK(cudaEventRecord(a, st->s));
    for (int r = 0; r < reps; ++r) CUDA_OK(cudaGraphLaunch(ex, st->s));
    CUDA_OK(cudaEventRecord(b, st->s));
    CUDA_OK(cudaEventSynchronize(b));
    float ms = 0.f;
    CUDA_OK(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaGraphExecDestroy(ex);
    *ms_per_rep = ms / reps;
    *launches_per_rep = st->gemv_launches;
    *bytes_per_rep = st->gemv_bytes;
    check_device_err(st);
  });
}

int mrtdf_bench_l2_read(mrtdf_engine* E, size_t bytes, int reps, double* gbs) {
  return guarded([&] {
    if (!E || !gbs || reps <= 0) throw Error{MRTDF_ERR_INVALID, "bad argument"};
    const size_t unit = (size_t)16 << 20;
    bytes = bytes / unit * unit;
    if (bytes == 0 || bytes > ((size_t)1 << 34)) throw Error{MRTDF_ERR_RANGE, "bytes must be in [16 MiB, 16 GiB]"};
    CUDA_OK(cudaSetDevice(E->device));
    uint8_t* buf = nullptr;
    unsigned* sink = nullptr;
    CUDA_OK(cudaMalloc(&buf, bytes));
    struct Free {
      void* a;
      void* b;
      ~Free() {
        cudaFree(a);
        cudaFree(b);
      }
    } fr{buf, nullptr};
    CUDA_OK(cudaMalloc(&sink, 4 * 4096));
    fr.b = sink;
    cudaStream_t s = nullptr;
    CUDA_OK(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    CUDA_OK(cudaMemsetAsync(buf, 1, bytes, s));
    check_cuda(launch_l2_read(buf, bytes, sink, E->num_sms, s), "l2 read");  // warm-up: the buffer lands in L2
    cudaEvent_t a, b;
    CUDA_OK(cudaEventCreate(&a));
    CUDA_OK(cudaEventCreate(&b));
    CUDA_OK(cudaEventRecord(a, s));
    for (int r = 0; r < reps; ++r) check_cuda(launch_l2_read(buf, bytes, sink, E->num_sms, s), "l2 read");
    CUDA_OK(cudaEventRecord(b, s));
    CUDA_OK(cudaEventSynchronize(b));
    float ms = 0.f;
    CUDA_OK(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaStreamDestroy(s);
    *gbs = (double)bytes * reps / (ms * 1e-3) / 1e9;
  });
}

int mrtdf_bench_encoder(mrtdf_engine* E, int rows, int seq_len, int reps, float* ms_per_rep, double* flops_per_rep) {
  return guarded([&] {
    if (!E || rows <= 0 || reps <= 0 || !ms_per_rep || !flops_per_rep) throw Error{MRTDF_ERR_INVALID, "bad argument"};
    if (!E->loaded) throw Error{MRTDF_ERR_STATE, "weights not loaded"};
    const mrtdf_config& c = E->c;
    if (seq_len <= 0 || seq_len > c.max_encoder_length) throw Error{MRTDF_ERR_RANGE, "seq_len out of range"};
    CUDA_OK(cudaSetDevice(E->device));
    // encoder-only workspace for `rows` sequences (no decode state)
    mrtdf_stream st;
    st.eng = E;
    st.nseq = rows;
    st.rps = 1;
    st.B = rows;
    CUDA_OK(cudaStreamCreateWithFlags(&st.s, cudaStreamNonBlocking));
    const size_t B = rows, d = c.d_model, in = E->inner(), ff = c.d_ff, H = c.num_heads, es = E->esize;
    const size_t M = B * seq_len;
    const size_t cross = (size_t)c.num_temporal_layers * B * H * c.max_encoder_length * 64 * es;
    std::vector<std::pair<void**, size_t>> plan = {
        {&st.ex, M * d * es}, {&st.en, M * d * es}, {&st.eqkv, M * 3 * in * es}, {&st.eo, M * in * es},
        {&st.eh, M * ff * es}, {(void**)&st.ids, M * 4}, {&st.ck, cross}, {&st.cv, cross}, {(void**)&st.err, 64}};
    size_t total = 0;
    for (auto& q : plan) total += (q.second + 255) & ~(size_t)255;
    st.mem.reserve(total);
    for (auto& q : plan) *q.first = st.mem.take(q.second);
    // uniform-random ids in [0, vocab), seed 2
    std::vector<int32_t> ids(M);
    uint64_t x = 2;
    for (auto& v : ids) {
      x += 0x9E3779B97F4A7C15ull;  // splitmix64
      uint64_t z = x;
      z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
      z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
      z ^= z >> 31;
      v = (int32_t)(z % (uint64_t)c.vocab_size);
    }
    CUDA_OK(cudaMemcpyAsync(st.ids, ids.data(), M * 4, cudaMemcpyHostToDevice, st.s));
    CUDA_OK(cudaMemsetAsync(st.err, 0, 64, st.s));
    st.S = seq_len;
    cudaGraph_t g = nullptr;
    CUDA_OK(cudaStreamBeginCapture(st.s, cudaStreamCaptureModeThreadLocal));
    try {
      enqueue_encode(&st, seq_len);
    } catch (...) {
      cudaStreamEndCapture(st.s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    CUDA_OK(cudaStreamEndCapture(st.s, &g));
    cudaGraphExec_t ex = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    check_cuda(e, "cudaGraphInstantiate");
    cudaEvent_t a, b;
    CUDA_OK(cudaEventCreate(&a));
    CUDA_OK(cudaEventCreate(&b));
    CUDA_OK(cudaGraphLaunch(ex, st.s));  // warm-up
    CUDA_OK(cudaEventRecord(a, st.s));
    for (int r = 0; r < reps; ++r) CUDA_OK(cudaGraphLaunch(ex, st.s));
    CUDA_OK(cudaEventRecord(b, st.s));
    CUDA_OK(cudaEventSynchronize(b));
    float ms = 0.f;
    CUDA_OK(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaGraphExecDestroy(ex);
    *ms_per_rep = ms / reps;
    // 2 flops per multiply-add: encoder linears, attention (QK^T and PV),
    // and the cross-K/V projection of every temporal layer
    const double Md = (double)M, S = seq_len;
    const double lin = 2.0 * Md * ((double)d * 3 * in + (double)in * d + (double)d * 2 * ff + (double)ff * d);
    const double att = 4.0 * (double)B * H * S * S * 64.0;
    *flops_per_rep = c.num_encoder_layers * (lin + att) + 2.0 * Md * d * (2.0 * c.num_temporal_layers * in);
    check_device_err(&st);
  });
}

int mrtdf_bench_depth(mrtdf_stream* st, const mrtdf_gen_opts* o, int frames, int reps, float* us_per_step,
                      double* bytes_per_step, long long* launches_per_step) {
  return guarded([&] {
    if (!st || !o || frames <= 0 || reps <= 0 || !us_per_step || !bytes_per_step || !launches_per_step)
      throw Error{MRTDF_ERR_INVALID, "bad argument"};
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    if (frames > c.max_frames) throw Error{MRTDF_ERR_RANGE, "frames must be <= max_frames"};
    if (o->rvq_depth != c.rvq_depth) throw Error{MRTDF_ERR_INVALID, "rvq_depth must equal the model's rvq_depth"};
    if (o->uniforms) throw Error{MRTDF_ERR_INVALID, "the depth microbenchmark draws with Philox"};
    CUDA_OK(cudaSetDevice(E->device));
    // one N(0, 1) temporal hidden state per frame and row (seed 3), in the compute dtype
    const size_t per_frame = (size_t)st->B * c.d_model;
    std::vector<float> xs(per_frame * frames);
    fill_random_tensor(3, 0, 1.0f, false, false, xs.data(), (int64_t)xs.size());
    const std::vector<uint8_t> xb = to_dtype(xs.data(), xs.size(), c.dtype);
    uint8_t* xd = nullptr;
    CUDA_OK(cudaMalloc(&xd, xb.size()));
    struct Free {
      uint8_t* p;
      ~Free() { cudaFree(p); }
    } free_xd{xd};
    CUDA_OK(cudaMemcpyAsync(xd, xb.data(), xb.size(), cudaMemcpyHostToDevice, st->s));
    upload_seeds(st, o, nullptr);
    const bool masked = o->use_vocab_masks != 0;
    st->gemv_launches = 0;
    st->gemv_bytes = 0.0;
    cudaGraph_t g = nullptr;
    CUDA_OK(cudaStreamBeginCapture(st->s, cudaStreamCaptureModeThreadLocal));
    try {
      fused_reset(st);
      for (int f = 0; f < frames; ++f)
        for (int l = 0; l < c.rvq_depth; ++l) {
          int lo, hi;
          level_range(c, masked, l, lo, hi);
          enqueue_depth(st, l, Hidden{l == 0 ? (const void*)(xd + act_bytes(E, per_frame * f)) : st->din, nullptr},
                        lo, hi);
          enqueue_sample(st, f, l, *o, masked, lo, hi, false);
        }
    } catch (...) {
      cudaStreamEndCapture(st->s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    CUDA_OK(cudaStreamEndCapture(st->s, &g));
    cudaGraphExec_t ex = nullptr;
    const cudaError_t e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    check_cuda(e, "cudaGraphInstantiate");
    cudaEvent_t a, b;
    CUDA_OK(cudaEventCreate(&a));
    CUDA_OK(cudaEventCreate(&b));
    CUDA_OK(cudaGraphLaunch(ex, st->s));  // warm-up
    CUDA_OK(cudaEventRecord(a, st->s));
    for (int r = 0; r < reps; ++r) CUDA_OK(cudaGraphLaunch(ex, st->s));
    CUDA_OK(cudaEventRecord(b, st->s));
    CUDA_OK(cudaEventSynchronize(b));
    float ms = 0.f;
    CUDA_OK(cudaEventElapsedTime(&ms, a, b));
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaGraphExecDestroy(ex);
    const double steps = (double)frames * c.rvq_depth;
    *us_per_step = (float)(ms * 1e3 / (reps * steps));
    // GEMV phases (weights, inputs, outputs) + the self-attention K/V reads
    double kv = 0.0;
    for (int l = 0; l < c.rvq_depth; ++l)
      kv += 2.0 * c.num_depth_layers * st->B * c.num_heads * (l + 1) * 64.0 * E->esize;
    *bytes_per_step = (st->gemv_bytes + kv * frames) / steps;
    // per level: layers x (self phase, FFN phase) + lm_head + sampler on the
    // fused path; else layers x (QKV, attention, o_proj, FFN-up, FFN-down)
    // with the attention inside the QKV launch for bf16 cluster attention
    const bool cl = c.dtype == MRTDF_DTYPE_BF16 && st->B <= kQkvCluster && E->cluster_attn;
    *launches_per_step = (long long)c.num_depth_layers * (st->fused ? 2 : cl ? 4 : 5) + 2;
    check_device_err(st);
  });
}


long long mrtdf_stream_chunk_kernels(const mrtdf_stream* st) { return st ? st->last_chunk_kernels : -1; }

// ---- single-layer probes -----------------------------------------------------
int mrtdf_probe_encoder_layer(mrtdf_stream* st, int layer, const float* x, int seq_len, float* out) {
  return guarded([&] {
    if (!st || !x || !out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    if (layer < 0 || layer >= c.num_encoder_layers) throw Error{MRTDF_ERR_RANGE, "encoder layer out of range"};
    if (seq_len <= 0 || seq_len > c.max_encoder_length) throw Error{MRTDF_ERR_RANGE, "seq_len out of range"};
    CUDA_OK(cudaSetDevice(E->device));
    const size_t n = (size_t)st->B * seq_len * c.d_model;
    float* tmp = nullptr;
    CUDA_OK(cudaMalloc(&tmp, n * 4));
    struct Free {
      float* p;
      ~Free() { cudaFree(p); }
    } free_tmp{tmp};
    CUDA_OK(cudaMemcpyAsync(tmp, x, n * 4, cudaMemcpyHostToDevice, st->s));
    check_cuda(launch_f32_to_act(c.dtype, tmp, n, st->ex, st->s), "convert");
    enqueue_encoder_layer(st, E->enc[layer], seq_len);
    check_cuda(launch_act_to_f32(c.dtype, st->ex, n, tmp, st->s), "convert");
    CUDA_OK(cudaMemcpyAsync(out, tmp, n * 4, cudaMemcpyDeviceToHost, st->s));
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
  });
}

int mrtdf_probe_set_cache(mrtdf_stream* st, int kind, int layer, const float* k, const float* v, int len) {
  return guarded([&] {
    if (!st || !k || !v) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    const int layers = kind == 1 ? c.num_depth_layers : c.num_temporal_layers;
    const int cap = kind == 0 ? c.max_frames : kind == 1 ? c.rvq_depth : c.max_encoder_length;
    if (kind < 0 || kind > 2 || layer < 0 || layer >= layers) throw Error{MRTDF_ERR_RANGE, "cache kind / layer"};
    if (len < 0 || len > cap || (kind == 2 && len == 0)) throw Error{MRTDF_ERR_RANGE, "cache length"};
    CUDA_OK(cudaSetDevice(E->device));
    const size_t rows_h = (size_t)st->B * c.num_heads, es = E->esize;
    const size_t per_layer = rows_h * cap * 64 * es;
    uint8_t* kd = (uint8_t*)(kind == 0 ? st->tk : kind == 1 ? st->dk : st->ck) + per_layer * layer;
    uint8_t* vd = (uint8_t*)(kind == 0 ? st->tv : kind == 1 ? st->dv : st->cv) + per_layer * layer;
    if (len > 0) {
      const size_t n = rows_h * len * 64;
      const std::vector<uint8_t> kb = to_dtype(k, n, c.dtype), vb = to_dtype(v, n, c.dtype);
      CUDA_OK(cudaMemcpy2DAsync(kd, cap * 64 * es, kb.data(), len * 64 * es, len * 64 * es, rows_h,
                                cudaMemcpyHostToDevice, st->s));
      CUDA_OK(cudaMemcpy2DAsync(vd, cap * 64 * es, vb.data(), len * 64 * es, len * 64 * es, rows_h,
                                cudaMemcpyHostToDevice, st->s));
      CUDA_OK(cudaStreamSynchronize(st->s));  // kb / vb are locals
    }
    if (kind == 2) {
      st->S = len;
      st->encoded = true;
    }
  });
}

int mrtdf_probe_decoder_layer(mrtdf_stream* st, int stack, int layer, int pos, const float* x, float* out) {
  return guarded([&] {
    if (!st || !x || !out) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    if (stack != 0 && stack != 1) throw Error{MRTDF_ERR_INVALID, "stack must be 0 (temporal) or 1 (depth)"};
    const int layers = stack == 0 ? c.num_temporal_layers : c.num_depth_layers;
    const int cap = stack == 0 ? c.max_frames : c.rvq_depth;
    if (layer < 0 || layer >= layers || pos < 0 || pos >= cap) throw Error{MRTDF_ERR_RANGE, "layer / pos"};
    if (stack == 0 && !st->encoded) throw Error{MRTDF_ERR_STATE, "temporal layer: no cross-attention cache"};
    CUDA_OK(cudaSetDevice(E->device));
    const size_t es = E->esize;
    if (stack == 0) {
      const size_t tcs = layer_cache_elems(st, c.max_frames), ccs = layer_cache_elems(st, c.max_encoder_length);
      upload_act(st, x, st->tin);
      void* tk = (uint8_t*)st->tk + tcs * es * layer;
      void* tv = (uint8_t*)st->tv + tcs * es * layer;
      const float* bias = E->tbias + (size_t)pos * c.num_heads * c.max_frames;
      const void* ck = (const uint8_t*)st->ck + ccs * es * layer;
      const void* cv = (const uint8_t*)st->cv + ccs * es * layer;
      if (st->fused) {
        fused_reset(st);
        materialize(st, enqueue_fused_layer(st, E->tl[layer], Hidden{st->tin, nullptr}, tk, tv, c.max_frames, pos,
                                            bias, c.max_frames, ck, cv, false),
                    st->tx);
      } else {
        enqueue_decoder_layer(st, E->tl[layer], st->tin, st->tx, tk, tv, c.max_frames, pos, bias, c.max_frames, ck,
                              cv, false);
      }
      download_act(st, st->tx, out);
    } else {
      const size_t dcs = layer_cache_elems(st, c.rvq_depth);
      upload_act(st, x, st->din);
      void* dk = (uint8_t*)st->dk + dcs * es * layer;
      void* dv = (uint8_t*)st->dv + dcs * es * layer;
      const float* bias = E->dbias + (size_t)pos * c.num_heads * c.rvq_depth;
      if (st->fused) {
        fused_reset(st);
        materialize(st, enqueue_fused_layer(st, E->dl[layer], Hidden{st->din, nullptr}, dk, dv, c.rvq_depth, pos,
                                            bias, c.rvq_depth, nullptr, nullptr, true),
                    st->dx);
      } else {
        enqueue_decoder_layer(st, E->dl[layer], st->din, st->dx, dk, dv, c.rvq_depth, pos, bias, c.rvq_depth,
                              nullptr, nullptr, true);
      }
      download_act(st, st->dx, out);
    }
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
  });
}

int mrtdf_probe_lm_head(mrtdf_stream* st, int level, const float* x, float* logits) {
  return guarded([&] {
    if (!st || !x || !logits) throw Error{MRTDF_ERR_INVALID, "NULL argument"};
    mrtdf_engine* E = st->eng;
    const mrtdf_config& c = E->c;
    if (level >= c.rvq_depth) throw Error{MRTDF_ERR_RANGE, "level out of range"};
    int lo, hi;
    level_range(c, level >= 0, level < 0 ? 0 : level, lo, hi);
    CUDA_OK(cudaSetDevice(E->device));
    upload_act(st, x, st->dx);
    GemvParams p{};
    p.W = (const uint8_t*)E->lm_head + act_bytes(E, (size_t)lo * c.d_model);
    p.x = st->dx; p.norm_w = E->dec_norm; p.out = st->logits; p.units = hi - lo; p.cols = c.d_model;
    p.x_stride = c.d_model; p.out_stride = c.vocab_size; p.out_offset = lo; p.l2_keep = 1;
    gemv(st, kGemvLogits, true, p);
    CUDA_OK(cudaMemcpy2DAsync(logits, (size_t)(hi - lo) * 4, st->logits + lo, (size_t)c.vocab_size * 4,
                              (size_t)(hi - lo) * 4, st->B, cudaMemcpyDeviceToHost, st->s));
    CUDA_OK(cudaStreamSynchronize(st->s));
    check_device_err(st);
  });
}

}  // extern "C"

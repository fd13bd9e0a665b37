// Model, compute handle and trunk sequencer behind the evaluator C ABI.
//
// Mirrors the reference's CUDA backend boundary (crates/kata_nn/src/backend.rs:
// 206-410, implemented by CudaBackend in src/backends/cuda.rs:2610-3105):
//   kb_model_load        ~ load_model_file + the deferred weight upload
//                          (cuda.rs:2618-2680, cuda_exec.rs:674-815, int8.rs:222)
//   kb_handle_create     ~ create_compute_handle (cuda.rs:2926): one stream,
//                          one workspace per physical batch, two pipeline slots
//   kb_submit / kb_query / kb_finish ~ submit_output / query_output_done /
//                          finish_output (cuda.rs:2196-2510): pinned staging,
//                          H2D, a CUDA graph per batch size, D2H, event wait,
//                          sticky status check before outputs are published
//   kb_forward_device    ~ CudaModel::apply (cuda_exec.rs:913) on device buffers
//
// The flat trunk (BASELINE b11c768 topology): stem (3x3 conv 22->C + global
// linear, one bf16 GEMM) -> num_blocks x [RMSNorm -> INT8 QKV GEMM -> RoPE
// attention -> INT8 out-proj + residual -> RMSNorm -> INT8 up GEMM + GELU ->
// INT8 down GEMM + residual] on a bf16 residual stream -> trunk tip (BN affine +
// SiLU) -> one bf16 GEMM for all per-token head linears -> policy/value heads.
//
// The nested trunk (the reference's TF3 graph, native_model.rs:79-124, run as
// cuda_exec.rs:1136-1700 runs it): stem as one binary16 GEMM into an fp32 raw
// trunk -> per outer block [gate-SiLU (pre_bn) -> binary16 C->mid linear into
// an fp32 inner stream -> pairs x (RMSNorm -> QKV (INT8 or binary16, RoPE in
// the epilogue) -> attention D32 -> out-proj + fp32 residual -> RMSNorm -> INT8
// SwiGLU FFN + fp32 residual) -> gate-SiLU (post_bn) -> binary16 mid->C linear
// added to the raw trunk] -> trunk tip -> heads.
#include <math.h>
#include <string.h>

#include <map>
#include <mutex>
#include <new>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/katab200.h"
#include "kb_handles.h"
#include "kb_internal.h"

namespace kb {
int attention_launch(const uint16_t* qkv, const float* rope_cos, const float* rope_sin, uint16_t* out,
                     int batch, int seq, int heads, int head_dim, float scale, int f16, cudaStream_t stream,
                     uint32_t* row_amax = nullptr, unsigned* status = nullptr);
int stem_gather_launch(const float* spatial, const float* global, const int* sym, uint16_t* a, int batch,
                       int nhwc, cudaStream_t s, int f16 = 0);
int gate_silu_launch(const float* x, long ldx, const float* scale, const float* bias, uint16_t* out, long ldo,
                     long rows, int w, int f16, cudaStream_t s);
int trunk_tip_launch(const uint16_t* x, const float* gamma, const float* beta, uint16_t* g, long rows, int c,
                     cudaStream_t s);
int heads_launch(const float* hp, const float* const* wts, float* policy, float* value, float* misc,
                 float* moremisc, float* ownership, int batch, unsigned* status, cudaStream_t s);
}  // namespace kb

using namespace kb;

namespace {

constexpr int kSide = 19;
constexpr int kSeq = 361;
constexpr int kInC = 22, kInG = 19;
constexpr int kStemK = 224, kStemKUsed = 217;
constexpr int kHeadN = 384;  // p1 96 | g1 96 | v1 192
constexpr float kRmsEps = 1e-6f;
constexpr int kNestedHeadDim = 32;  // native_model.rs:15 (DIM)

// Host-side view of the fp32 weight blob (layout documented in katab200.h).
struct BlobCursor {
  const float* p;
  size_t left;
  const float* take(size_t n) {
    if (n > left) return nullptr;
    const float* r = p;
    p += n;
    left -= n;
    return r;
  }
};

size_t blob_floats(const kb_model_desc& d) {
  const size_t c = d.trunk_channels, f = d.ffn_channels, h = d.num_heads, hd = d.head_dim;
  size_t n = c * kStemKUsed;
  if (d.topology == KB_TOPO_NESTED) {
    const size_t m = d.mid_channels;
    const size_t pair = m + 3 * m * m + m * m + h * (hd / 2) * 2 + m + 2 * f * m + m * f;
    n += d.num_blocks * (2 * c + m * c + d.pairs_per_block * pair + 2 * m + c * m);
  } else {
    n += d.num_blocks * (c + 3 * c * c + c * c + c + f * c + f + c * f + c + h * (hd / 2) * 2);
  }
  n += 2 * c;
  n += 96 * c + 96 * c + 96 + 192 * c + 192;
  n += 96 * 288 + 96 * 288 + 96 + 6 * 96 + 96 + 6 * 96;
  n += 192 * 576 + 192 + 3 * 192 + 3 + 10 * 192 + 10 + 8 * 192 + 8 + 192;
  return n;
}

int validate_nested(const kb_model_desc* d) {
  const int m = d->mid_channels, h = d->ffn_channels;
  // native_model.rs:31-60, :91-104 (D = 32, SwiGLU hidden <= 3*mid, 8-aligned),
  // plus this build's GEMM tiling (C % 64, mid % 32).
  if (d->trunk_channels <= 0 || d->trunk_channels % 64 != 0 || d->trunk_channels > 4096 || m < 32 ||
      m % 32 != 0 || m >= d->trunk_channels || m > 2048 || d->num_blocks <= 0 || d->num_blocks > 64 ||
      d->pairs_per_block < 1 || d->pairs_per_block > 8 || d->head_dim != kNestedHeadDim ||
      d->num_heads * kNestedHeadDim != m || h <= 0 || h % 8 != 0 || h > 3 * m ||
      !(d->norm_eps >= 0.0f) || !std::isfinite(d->norm_eps)) {
    set_error("nested model descriptor: need C % 64 == 0 (<= 4096), 32 <= mid < C with mid % 32 == 0, "
              "heads * 32 == mid (head_dim 32), SwiGLU hidden 8-aligned and <= 3*mid, 1..64 outer blocks of "
              "1..8 pairs, a finite epsilon >= 0");
    return KB_E_INVALID;
  }
  if (d->precision != KB_PREC_INT8) {
    set_error("nested model descriptor: precision must be KB_PREC_INT8 (INT8 SwiGLU FFN)");
    return KB_E_INVALID;
  }
  for (int i = 0; i < 4; ++i) {
    const int p = d->proj_precision[i];
    const bool ok = i < KB_PROJ_FFN_UP ? (p == KB_PROJ_FOLLOW || p == KB_PROJ_INT8 || p == KB_PROJ_BF16)
                                       : (p == KB_PROJ_FOLLOW || p == KB_PROJ_INT8);
    if (!ok) {
      set_error("nested model descriptor: qkv / out projections INT8 or 16-bit (KB_PROJ_BF16 = binary16 here), "
                "the SwiGLU FFN INT8");
      return KB_E_INVALID;
    }
  }
  if (d->int8_min_ffn_width < 0 || d->int8_min_ffn_width > 8192 || d->int8_min_ffn_width % 8 != 0 ||
      (d->int8_min_ffn_width > 0 && h < d->int8_min_ffn_width)) {
    set_error("nested model descriptor: int8_min_ffn_width would leave the SwiGLU FFN unquantised, which the "
              "nested path does not run");
    return KB_E_INVALID;
  }
  return KB_OK;
}

int validate_desc(const kb_model_desc* d) {
  if (d && d->topology == KB_TOPO_NESTED) return validate_nested(d);
  if (d && (d->topology != KB_TOPO_FLAT || !(d->norm_eps >= 0.0f) || !std::isfinite(d->norm_eps))) {
    set_error("model descriptor: topology must be KB_TOPO_FLAT or KB_TOPO_NESTED, norm_eps finite and >= 0");
    return KB_E_INVALID;
  }
  if (!d || d->trunk_channels <= 0 || d->trunk_channels % 64 != 0 || d->trunk_channels > 4096 ||
      d->num_blocks <= 0 || d->num_blocks > 64 || d->num_heads <= 0 ||
      (d->head_dim != 32 && d->head_dim != 64) || d->num_heads * d->head_dim != d->trunk_channels ||
      d->ffn_channels <= 0 || d->ffn_channels % 64 != 0 || d->ffn_channels > 4096 ||
      (d->precision != KB_PREC_INT8 && d->precision != KB_PREC_MXFP8)) {
    set_error("model descriptor: need C % 64 == 0 (<= 4096), heads*head_dim == C, head_dim 32|64, "
              "F % 64 == 0 (<= 4096), 1..64 blocks, precision KB_PREC_INT8 or KB_PREC_MXFP8");
    return KB_E_INVALID;
  }
  for (int i = 0; i < 4; ++i)
    if (d->proj_precision[i] < KB_PROJ_FOLLOW || d->proj_precision[i] > KB_PROJ_BF16) {
      set_error("model descriptor: proj_precision entries must be KB_PROJ_FOLLOW, _INT8, _MXFP8 or _BF16");
      return KB_E_INVALID;
    }
  // parse_min_ffn_width (crates/kata_nn/src/backends/int8.rs:75-83)
  if (d->int8_min_ffn_width < 0 || d->int8_min_ffn_width > 8192 || d->int8_min_ffn_width % 8 != 0) {
    set_error("model descriptor: int8_min_ffn_width must be 8-aligned and in 0..=8192");
    return KB_E_INVALID;
  }
  return KB_OK;
}

// Each projection's precision (KB_PROJ_INT8 / _MXFP8 / _BF16) for qkv, out,
// ffn_up, ffn_down: the recipe's entry, else the model's precision; an INT8
// FFN projection narrower than int8_min_ffn_width stays unquantised, as the
// reference's selective INT8 load keeps it in FP16 (cuda_exec.rs:631-690).
void resolve_precision(const kb_model_desc& d, int (&out)[4]) {
  const int base = d.precision == KB_PREC_MXFP8 ? KB_PROJ_MXFP8 : KB_PROJ_INT8;
  for (int i = 0; i < 4; ++i) {
    int p = d.proj_precision[i] ? d.proj_precision[i] : base;
    if (i >= KB_PROJ_FFN_UP && p == KB_PROJ_INT8 && d.int8_min_ffn_width > 0 &&
        d.ffn_channels < d.int8_min_ffn_width)
      p = KB_PROJ_BF16;
    out[i] = p;
  }
}

template <typename T>
int dev_alloc(T** p, size_t count, const char* what) {
  return check_cuda(cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T) + 16), what);
}

template <typename T>
int upload(T** dst, const T* src, size_t count, const char* what) {
  int rc = dev_alloc(dst, count, what);
  if (rc) return rc;
  return check_cuda(cudaMemcpy(*dst, src, count * sizeof(T), cudaMemcpyHostToDevice), what);
}

uint16_t bf16_bits(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  if ((b & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>(((b >> 16) & 0x8000u) | 0x7fc0u);
  b += 0x7fffu + ((b >> 16) & 1u);
  return static_cast<uint16_t>(b >> 16);
}

// IEEE binary16 round-to-nearest-even of a finite float (host).
uint16_t f16_bits(float v) {
  uint32_t b;
  memcpy(&b, &v, 4);
  const uint16_t sign = static_cast<uint16_t>((b >> 16) & 0x8000u);
  const int e = static_cast<int>((b >> 23) & 255u) - 127 + 15;
  uint32_t mant = b & 0x7fffffu;
  if (e >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return sign;
    mant |= 0x800000u;
    const uint32_t shift = static_cast<uint32_t>(14 - e);
    uint32_t r = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (r & 1u))) ++r;
    return static_cast<uint16_t>(sign | r);
  }
  uint32_t r = mant >> 13;
  const uint32_t rem = mant & 0x1fffu;
  uint32_t ex = static_cast<uint32_t>(e);
  if (rem > 0x1000u || (rem == 0x1000u && (r & 1u))) {
    if (++r == 0x400u) {
      r = 0;
      if (++ex >= 31) return static_cast<uint16_t>(sign | 0x7c00u);
    }
  }
  return static_cast<uint16_t>(sign | (ex << 10) | r);
}

uint16_t bits16(float v, bool f16) { return f16 ? f16_bits(v) : bf16_bits(v); }

// Rotary tables of one attention layer: angle = x*f0 + y*f1 in fp32, cosf /
// sinf (native_model.rs:200-228), laid out [head * pairs + pair, token] so the
// QKV epilogue's 32 consecutive rows (tokens) read one contiguous run.
int upload_rope(const float* freqs, int nh, int hd, float** cos_d, float** sin_d) {
  const int pairs = hd / 2;
  std::vector<float> cs(static_cast<size_t>(kSeq) * nh * pairs), sn(cs.size());
  for (int y = 0; y < kSide; ++y)
    for (int x = 0; x < kSide; ++x)
      for (int hh = 0; hh < nh; ++hh)
        for (int p = 0; p < pairs; ++p) {
          const int fi = (hh * pairs + p) * 2;
          const float angle = static_cast<float>(x) * freqs[fi] + static_cast<float>(y) * freqs[fi + 1];
          const size_t idx = (static_cast<size_t>(hh) * pairs + p) * kSeq + (y * kSide + x);
          cs[idx] = cosf(angle);
          sn[idx] = sinf(angle);
        }
  int rc = upload(cos_d, cs.data(), cs.size(), "upload rope");
  if (!rc) rc = upload(sin_d, sn.data(), sn.size(), "upload rope");
  return rc;
}

// A weight [n, k] as binary16 on the device.
int upload_f16(uint16_t** dst, const float* w, size_t count) {
  std::vector<uint16_t> hw(count);
  for (size_t i = 0; i < count; ++i) hw[i] = f16_bits(w[i]);
  return upload(dst, hw.data(), hw.size(), "upload binary16 weight");
}

struct Block {
  float* rms1 = nullptr;
  float* rms2 = nullptr;
  kb_int8_weight* qkv = nullptr;
  kb_int8_weight* out = nullptr;
  kb_int8_weight* up = nullptr;
  kb_int8_weight* down = nullptr;
  // KB_PREC_MXFP8: the same four projections as block-scaled E4M3 weights.
  kb_mxfp8_weight* mqkv = nullptr;
  kb_mxfp8_weight* mout = nullptr;
  kb_mxfp8_weight* mup = nullptr;
  kb_mxfp8_weight* mdown = nullptr;
  // KB_PROJ_BF16 projections: bf16-rounded weights [N, K].
  uint16_t* bqkv = nullptr;
  uint16_t* bout = nullptr;
  uint16_t* bup = nullptr;
  uint16_t* bdown = nullptr;
  float* up_b = nullptr;
  float* down_b = nullptr;
  float* rope_cos = nullptr;  // [361, heads, head_dim/2]
  float* rope_sin = nullptr;
};

// One attention / FFN pair of a nested outer block.
struct NestedPair {
  float* rms1 = nullptr;
  float* rms2 = nullptr;
  kb_int8_weight* qkv = nullptr;  // INT8 projections, or
  kb_int8_weight* out = nullptr;
  uint16_t* hqkv = nullptr;       // binary16 [3M, M] / [M, M]
  uint16_t* hout = nullptr;
  kb_int8_weight* dual = nullptr;  // SwiGLU [gate; up] [2H, M], tile-interleaved
  kb_int8_weight* down = nullptr;  // [M, H]
  float* rope_cos = nullptr;       // [heads * 16 + pair, token]
  float* rope_sin = nullptr;
};

struct NestedBlock {
  float* pre_s = nullptr;  // pre_bn scale / bias [C]
  float* pre_b = nullptr;
  uint16_t* pre_w = nullptr;  // binary16 [M, C]
  std::vector<NestedPair> pairs;
  float* post_s = nullptr;  // post_bn scale / bias [M]
  float* post_b = nullptr;
  uint16_t* post_w = nullptr;  // binary16 [C, M]
};

}  // namespace

struct kb_model {
  kb_model_desc desc{};
  float eps = kRmsEps;  // RMSNorm epsilon
  std::vector<NestedBlock> nblocks;  // KB_TOPO_NESTED
  int prec[4] = {};    // resolved KB_PROJ_* of qkv, out, ffn_up, ffn_down
  bool mixed = false;  // not every projection in the model's `precision`
  int device = 0;
  uint16_t* stem_w = nullptr;  // bf16 [C, 224]
  std::vector<Block> blocks;
  float* tip_gamma = nullptr;
  float* tip_beta = nullptr;
  uint16_t* head_w = nullptr;  // bf16 [384, C]
  float* head_b = nullptr;     // [384]
  float* small = nullptr;      // all small head weights, one allocation
  const float* head_ptrs[15] = {};
};

namespace {

struct Slot {
  float* h_spatial = nullptr;  // pinned
  float* h_global = nullptr;  // [n, 19] global features, then n int32 symmetries
  float* h_out = nullptr;      // pinned [policy | value | misc | moremisc | ownership]
  float* d_spatial = nullptr;
  float* d_global = nullptr;
  float* d_out = nullptr;
  unsigned* h_status = nullptr;  // pinned copy of the status word
  // kb_submit_rows: [row params n x 24 B | legality n x 362 B], and the decoded outputs.
  uint8_t* h_post = nullptr;
  uint8_t* d_post = nullptr;
  float* h_dec = nullptr;
  float* d_dec = nullptr;
  cudaEvent_t done = nullptr;
  cudaEvent_t inputs_ready = nullptr;  // this slot's host-to-device copies landed
  int n = 0;
  bool busy = false;
  bool decoded = false;
  uint64_t token = 0;
};

constexpr int kOutPerPos = 6 * 362 + 3 + 10 + 8 + 361;
constexpr int kDecPerPos = 362 + 3 + 4 + 2 + 361;
constexpr int kPostPerPos = static_cast<int>(sizeof(kb_row_params)) + 362;
static_assert(sizeof(kb_row_params) == 24, "kb_row_params is 24 bytes");
static_assert(sizeof(kb_postprocess_params) == 64, "kb_postprocess_params is 64 bytes");

}  // namespace

struct kb_handle {
  kb_model* model = nullptr;
  int device = 0;
  int max_batch = 0;
  int nhwc = 0;
  cudaStream_t stream = nullptr;
  // Host-to-device input copies of kb_submit / kb_submit_rows: a second
  // submission's copies overlap the forward of the one in flight.
  cudaStream_t copy_stream = nullptr;
  // workspace
  uint16_t* stem_a = nullptr;   // [M, 224] bf16
  uint16_t* x = nullptr;        // [M, C] residual
  uint16_t* qkv = nullptr;      // [M, 3C]
  uint16_t* att = nullptr;      // [M, C] (also the trunk-tip output)
  uint16_t* hidden = nullptr;   // [M, F]
  int8_t* q = nullptr;          // [M, max kp] int8 or E4M3 bytes
  float* scales = nullptr;      // [M]
  uint8_t* mx_scales = nullptr; // MXFP8 packed UE8M0 scales for [M, max kp]
  size_t mx_scale_bytes = 0;
  uint32_t* row_amax = nullptr; // [M] |bits| maximum of the FFN hidden rows
  float* hp = nullptr;          // [M, 384] fp32
  float* x32 = nullptr;         // nested: raw trunk [M, C] fp32
  float* mid32 = nullptr;       // nested: inner stream [M, mid] fp32
  unsigned* status = nullptr;   // [2]
  kb_postprocess_params pp = kb::default_postprocess_params();
  Slot slots[2];
  uint64_t next_token = 1;
  // Graphs bake in buffer addresses: one per (batch size, input, symmetry and output buffers).
  using GraphKey = std::tuple<int, const void*, const void*, const void*, const void*>;
  std::map<GraphKey, cudaGraphExec_t> graphs;
  std::map<GraphKey, int> warmed;
  std::mutex mu;
};

namespace {

void destroy_model(kb_model* m) {
  if (!m) return;
  cudaFree(m->stem_w);
  for (auto& b : m->blocks) {
    cudaFree(b.rms1);
    cudaFree(b.rms2);
    kb_int8_weight_destroy(b.qkv);
    kb_int8_weight_destroy(b.out);
    kb_int8_weight_destroy(b.up);
    kb_int8_weight_destroy(b.down);
    kb_mxfp8_weight_destroy(b.mqkv);
    kb_mxfp8_weight_destroy(b.mout);
    kb_mxfp8_weight_destroy(b.mup);
    kb_mxfp8_weight_destroy(b.mdown);
    cudaFree(b.bqkv);
    cudaFree(b.bout);
    cudaFree(b.bup);
    cudaFree(b.bdown);
    cudaFree(b.up_b);
    cudaFree(b.down_b);
    cudaFree(b.rope_cos);
    cudaFree(b.rope_sin);
  }
  for (auto& nb : m->nblocks) {
    cudaFree(nb.pre_s);
    cudaFree(nb.pre_b);
    cudaFree(nb.pre_w);
    cudaFree(nb.post_s);
    cudaFree(nb.post_b);
    cudaFree(nb.post_w);
    for (auto& pr : nb.pairs) {
      cudaFree(pr.rms1);
      cudaFree(pr.rms2);
      kb_int8_weight_destroy(pr.qkv);
      kb_int8_weight_destroy(pr.out);
      cudaFree(pr.hqkv);
      cudaFree(pr.hout);
      kb_int8_weight_destroy(pr.dual);
      kb_int8_weight_destroy(pr.down);
      cudaFree(pr.rope_cos);
      cudaFree(pr.rope_sin);
    }
  }
  cudaFree(m->tip_gamma);
  cudaFree(m->tip_beta);
  cudaFree(m->head_w);
  cudaFree(m->head_b);
  cudaFree(m->small);
  delete m;
}

// The QKV projection rotates Q and K in its epilogue (learned 2-D RoPE tables
// [token, head, pair], native_model.rs:200-228): the rotation is applied to the
// fp32 projection before the bf16 rounding, and attention reads rotated Q/K.
void set_rope(GemmArgs& g, const Block& b, const kb_model_desc& d) {
  g.rope_cos = b.rope_cos;
  g.rope_sin = b.rope_sin;
  g.rope_cols = 2 * d.trunk_channels;
  g.rope_heads = d.num_heads;
  g.rope_hd = d.head_dim;
  g.rope_seq = kSeq;
}

// GemmArgs of one MXFP8 projection of the trunk (bf16 output or residual).
GemmArgs mx_args(kb_handle* h, const kb_mxfp8_weight* w, int M, void* out, const float* bias, int act,
                 unsigned layer) {
  GemmArgs g;
  g.m = M;
  g.n = w->n;
  g.k = w->kp;
  g.out = out;
  g.ldo = w->n;
  g.bias = bias;
  g.act = act;
  g.out_f16 = 0;
  g.status = h->status;
  g.layer = layer;
  g.sfa = h->mx_scales;
  g.sfb = w->scales;
  return g;
}

// One transformer block with MXFP8 projections (KB_PREC_MXFP8):
// RMSNorm -> MXFP8 -> QKV GEMM (bf16) -> RoPE attention -> MXFP8 -> out-proj +
// residual -> RMSNorm -> MXFP8 -> up GEMM + bias + GELU (bf16) -> MXFP8 ->
// down GEMM + bias + residual.  Every activation quantiser is the block-32
// E4M3/UE8M0 quantiser of the reference's MXFP8 path (mxfp8.cu:36-79) applied
// to the 16-bit boundary, as Mxfp8Workspace::project does (mxfp8.rs:1055-1121).
int mxfp8_block(kb_handle* h, const Block& b, unsigned layer, int n, float scale, uint16_t* trace_att) {
  const kb_model_desc& d = h->model->desc;
  const int c = d.trunk_channels, f = d.ffn_channels, M = n * kSeq;
  cudaStream_t s = h->stream;
  uint8_t* q = reinterpret_cast<uint8_t*>(h->q);
  int rc = rms_mxfp8_launch(h->x, KB_DT_BF16, c, M, c, b.rms1, h->model->eps, 0, q, h->mx_scales, h->status, layer, s);
  if (!rc) {
    GemmArgs gq = mx_args(h, b.mqkv, M, h->qkv, nullptr, 0, layer);
    set_rope(gq, b, d);
    rc = gemm_launch(kGemmMXF8, kEpiRope16, q, b.mqkv->q, gq, s);
  }
  if (!rc)
    rc = attention_launch(h->qkv, nullptr, nullptr, h->att, n, kSeq, d.num_heads, d.head_dim, scale, 0, s, nullptr,
                          h->status);
  if (!rc && trace_att)
    rc = check_cuda(cudaMemcpyAsync(trace_att, h->att, static_cast<size_t>(M) * c * 2, cudaMemcpyDeviceToDevice, s),
                    "trace copy");
  // Quantiser scale capacity = this shape's bytes: no tail clear inside the forward.
  size_t sb_c = 0, sb_f = 0;
  if (!rc) rc = mxfp8_dims(M, c, nullptr, nullptr, nullptr, &sb_c);
  if (!rc) rc = mxfp8_dims(M, f, nullptr, nullptr, nullptr, &sb_f);
  if (!rc)
    rc = mxfp8_quantize_launch(h->att, KB_DT_BF16, c, M, c, q, h->mx_scales, sb_c, false, h->status, layer, s);
  if (!rc) rc = gemm_launch(kGemmMXF8, kEpiRes16, q, b.mout->q, mx_args(h, b.mout, M, h->x, nullptr, 0, layer), s);
  if (!rc) rc = rms_mxfp8_launch(h->x, KB_DT_BF16, c, M, c, b.rms2, h->model->eps, 0, q, h->mx_scales, h->status, layer, s);
  if (!rc)
    rc = gemm_launch(kGemmMXF8, kEpi16, q, b.mup->q, mx_args(h, b.mup, M, h->hidden, b.up_b, KB_ACT_GELU, layer), s);
  if (!rc)
    rc = mxfp8_quantize_launch(h->hidden, KB_DT_BF16, f, M, f, q, h->mx_scales, sb_f, false, h->status, layer, s);
  if (!rc)
    rc = gemm_launch(kGemmMXF8, kEpiRes16, q, b.mdown->q, mx_args(h, b.mdown, M, h->x, b.down_b, 0, layer), s);
  return rc;
}

// ---- Mixed per-projection precision (a precision recipe) ----------------

int gemm_kind_of(int prec) {
  return prec == KB_PROJ_INT8 ? kGemmI8 : prec == KB_PROJ_MXFP8 ? kGemmMXF8 : kGemmBF16;
}

// The A operand of a projection of precision `prec` from bf16 rows src [M, k]:
// INT8 -> h->q + h->scales, MXFP8 -> h->q + h->mx_scales (with the RMSNorm
// fused when gamma is set), BF16 -> the rows themselves, or their RMSNorm in
// h->att.  The same quantisers as the single-precision blocks.
int mixed_operand(kb_handle* h, int prec, const uint16_t* src, int M, int k, int kp, const float* gamma,
                  unsigned layer, const void** a) {
  cudaStream_t s = h->stream;
  uint8_t* q8 = reinterpret_cast<uint8_t*>(h->q);
  if (prec == KB_PROJ_INT8) {
    *a = h->q;
    return quantize_rows_launch(src, KB_DT_BF16, k, M, k, kp, gamma != nullptr, gamma, h->model->eps, 0, h->q,
                                h->scales,
                                h->status, layer, s);
  }
  if (prec == KB_PROJ_MXFP8) {
    *a = q8;
    if (gamma)
      return rms_mxfp8_launch(src, KB_DT_BF16, k, M, k, gamma, h->model->eps, 0, q8, h->mx_scales, h->status, layer,
                              s);
    size_t sb = 0;
    int rc = mxfp8_dims(M, k, nullptr, nullptr, nullptr, &sb);
    if (!rc) rc = mxfp8_quantize_launch(src, KB_DT_BF16, k, M, k, q8, h->mx_scales, sb, false, h->status, layer, s);
    return rc;
  }
  if (!gamma) {
    *a = src;
    return KB_OK;
  }
  *a = h->att;
  return rms16_rows_launch(src, KB_DT_BF16, k, M, k, gamma, h->model->eps, 0, h->att, k, h->status, layer, s);
}

// One projection out[M, n] of the mixed block in its precision.
int mixed_gemm(kb_handle* h, int prec, const void* a, const kb_int8_weight* wi, const kb_mxfp8_weight* wm,
               const uint16_t* wb, int M, int n, int k, int epi, void* out, const float* bias, int act, unsigned layer,
               const Block* rope_block) {
  GemmArgs g;
  const void* bw = nullptr;
  if (prec == KB_PROJ_MXFP8) {
    g = mx_args(h, wm, M, out, bias, act, layer);
    bw = wm->q;
  } else {
    g.m = M;
    g.n = n;
    g.out = out;
    g.ldo = n;
    g.bias = bias;
    g.act = act;
    g.out_f16 = 0;
    g.status = h->status;
    g.layer = layer;
    if (prec == KB_PROJ_INT8) {
      g.k = wi->kp;
      g.row_scale = h->scales;
      g.col_scale = wi->scales;
      bw = wi->q;
    } else {
      g.k = k;
      bw = wb;
    }
  }
  if (rope_block) set_rope(g, *rope_block, h->model->desc);
  return gemm_launch(gemm_kind_of(prec), epi, a, bw, g, h->stream);
}

// One transformer block whose four projections each run in their own
// precision (kb_model::prec): the single-precision blocks' sequence, with each
// projection's input quantised (or not) for its own precision.
int mixed_block(kb_handle* h, const Block& b, unsigned layer, int n, float scale, uint16_t* trace_att) {
  const kb_model* m = h->model;
  const kb_model_desc& d = m->desc;
  const int c = d.trunk_channels, f = d.ffn_channels, M = n * kSeq;
  const int kpc = (c + 15) / 16 * 16, kpf = (f + 15) / 16 * 16;
  cudaStream_t s = h->stream;
  const void* a = nullptr;
  int rc = mixed_operand(h, m->prec[KB_PROJ_QKV], h->x, M, c, kpc, b.rms1, layer, &a);
  if (!rc)
    rc = mixed_gemm(h, m->prec[KB_PROJ_QKV], a, b.qkv, b.mqkv, b.bqkv, M, 3 * c, c, kEpiRope16, h->qkv, nullptr, 0,
                    layer, &b);
  if (!rc)
    rc = attention_launch(h->qkv, nullptr, nullptr, h->att, n, kSeq, d.num_heads, d.head_dim, scale, 0, s, nullptr,
                          h->status);
  if (!rc && trace_att)
    rc = check_cuda(cudaMemcpyAsync(trace_att, h->att, static_cast<size_t>(M) * c * 2, cudaMemcpyDeviceToDevice, s),
                    "trace copy");
  if (!rc) rc = mixed_operand(h, m->prec[KB_PROJ_OUT], h->att, M, c, kpc, nullptr, layer, &a);
  if (!rc)
    rc = mixed_gemm(h, m->prec[KB_PROJ_OUT], a, b.out, b.mout, b.bout, M, c, c, kEpiRes16, h->x, nullptr, 0, layer,
                    nullptr);
  if (!rc) rc = mixed_operand(h, m->prec[KB_PROJ_FFN_UP], h->x, M, c, kpc, b.rms2, layer, &a);
  if (!rc)
    rc = mixed_gemm(h, m->prec[KB_PROJ_FFN_UP], a, b.up, b.mup, b.bup, M, f, c, kEpi16, h->hidden, b.up_b,
                    KB_ACT_GELU, layer, nullptr);
  if (!rc) rc = mixed_operand(h, m->prec[KB_PROJ_FFN_DOWN], h->hidden, M, f, kpf, nullptr, layer, &a);
  if (!rc)
    rc = mixed_gemm(h, m->prec[KB_PROJ_FFN_DOWN], a, b.down, b.mdown, b.bdown, M, c, f, kEpiRes16, h->x, b.down_b, 0,
                    layer, nullptr);
  return rc;
}

// ---- nested (TF3) trunk --------------------------------------------------

// The attention scale of the lowered TF3 graph: qk_scale = 1 / sqrt(sqrt(32))
// applied to both q and k (native_model.rs:195), i.e. qk_scale^2 on q.k
// (cuda_exec.rs:1294), each step rounded to fp32.
float nested_attention_scale() {
  const float qk = 1.0f / sqrtf(sqrtf(static_cast<float>(kNestedHeadDim)));
  return qk * qk;
}

// A binary16 tensor-core GEMM with an fp32 result: out[M, n] = a . w^T, plus
// the fp32 `residual` (may alias out) when given.
int f16_gemm_f32(kb_handle* h, const uint16_t* a, const uint16_t* w, int M, int n, int k, float* out,
                 const float* residual) {
  GemmArgs g;
  g.m = M;
  g.n = n;
  g.k = k;
  g.out = out;
  g.ldo = n;
  g.residual = const_cast<float*>(residual);
  g.ldr = n;
  g.ab_f16 = 1;
  g.status = h->status;
  return gemm_launch(kGemmBF16, kEpiF32, a, w, g, h->stream);
}

// One attention / FFN pair on the fp32 inner stream h->mid32 [M, mid]:
// RMSNorm -> QKV (INT8 with the fused RMS quantiser, or binary16 on the
// RMSNorm's binary16 rows) with RoPE in the epilogue -> attention (binary16
// P) -> out-proj added to the fp32 stream (INT8 dequant-residual, or binary16
// GEMM + residual) -> RMSNorm -> INT8 dual GEMM + SwiGLU (fp16 boundaries,
// row |max| from the epilogue) -> one-pass requant -> INT8 down GEMM added to
// the fp32 stream: the reference's
// Int8Workspace::ffn_rms (int8.rs:1135-1172).
int nested_pair(kb_handle* h, const NestedPair& p, unsigned layer, int n, float scale) {
  const kb_model* m = h->model;
  const kb_model_desc& d = m->desc;
  const int mid = d.mid_channels, hid = d.ffn_channels, M = n * kSeq;
  cudaStream_t s = h->stream;
  int rc;
  GemmArgs g;
  g.m = M;
  g.n = 3 * mid;
  g.out = h->qkv;
  g.ldo = 3 * mid;
  g.out_f16 = 1;
  g.status = h->status;
  g.layer = layer;
  g.rope_cos = p.rope_cos;
  g.rope_sin = p.rope_sin;
  g.rope_cols = 2 * mid;
  g.rope_heads = d.num_heads;
  g.rope_hd = kNestedHeadDim;
  g.rope_seq = kSeq;
  if (p.qkv) {
    rc = quantize_rows_launch(h->mid32, KB_DT_F32, mid, M, mid, p.qkv->kp, true, p.rms1, m->eps, 1, h->q, h->scales,
                              h->status, layer, s);
    if (rc) return rc;
    g.k = p.qkv->kp;
    g.row_scale = h->scales;
    g.col_scale = p.qkv->scales;
    rc = gemm_launch(kGemmI8, kEpiRope16, h->q, p.qkv->q, g, s);
  } else {
    rc = rms16_rows_launch(h->mid32, KB_DT_F32, mid, M, mid, p.rms1, m->eps, 1, h->att, mid, h->status, layer, s);
    if (rc) return rc;
    g.k = mid;
    g.ab_f16 = 1;
    rc = gemm_launch(kGemmBF16, kEpiRope16, h->att, p.hqkv, g, s);
  }
  if (rc) return rc;
  if (p.out) {
    rc = check_cuda(cudaMemsetAsync(h->row_amax, 0, static_cast<size_t>(M) * sizeof(uint32_t), s), "amax reset");
    if (rc) return rc;
  }
  rc = attention_launch(h->qkv, nullptr, nullptr, h->att, n, kSeq, d.num_heads, kNestedHeadDim, scale, 1, s,
                        p.out ? h->row_amax : nullptr, h->status);
  if (rc) return rc;
  if (p.out) {
    rc = quantize_rows_amax_launch(h->att, KB_DT_F16, mid, h->row_amax, M, mid, p.out->kp, h->q, h->scales, h->status,
                                   layer, s);
    if (rc) return rc;
    GemmArgs o;
    o.m = M;
    o.n = mid;
    o.k = p.out->kp;
    o.out = h->mid32;
    o.ldo = mid;
    o.row_scale = h->scales;
    o.col_scale = p.out->scales;
    o.status = h->status;
    o.layer = layer;
    rc = gemm_launch(kGemmI8, kEpiResF32, h->q, p.out->q, o, s);
  } else {
    rc = f16_gemm_f32(h, h->att, p.hout, M, mid, mid, h->mid32, h->mid32);
  }
  if (rc) return rc;
  // SwiGLU FFN: RMSNorm -> fp16 boundary -> INT8 -> dual GEMM + SwiGLU -> requant -> down + fp32 residual
  rc = quantize_rows_launch(h->mid32, KB_DT_F32, mid, M, mid, p.dual->kp, true, p.rms2, m->eps, 1, h->q, h->scales,
                            h->status, layer, s);
  if (rc) return rc;
  GemmArgs u;
  u.m = M;
  u.n = p.dual->n_stored;
  u.k = p.dual->kp;
  u.out = h->hidden;
  u.ldo = hid;
  u.row_scale = h->scales;
  u.col_scale = p.dual->scales;
  u.out_f16 = 1;
  u.n_out = hid;
  u.status = h->status;
  u.layer = layer;
  // the epilogue emits each row's |max| so the requantiser needs one pass
  u.row_amax = h->row_amax;
  rc = check_cuda(cudaMemsetAsync(h->row_amax, 0, static_cast<size_t>(M) * sizeof(uint32_t), s), "amax reset");
  if (rc) return rc;
  rc = gemm_launch(kGemmI8, kEpiSwiGLU16, h->q, p.dual->q, u, s, 256);
  if (rc) return rc;
  rc = quantize_rows_amax_launch(h->hidden, KB_DT_F16, hid, h->row_amax, M, hid, p.down->kp, h->q, h->scales,
                                 h->status, layer, s);
  if (rc) return rc;
  GemmArgs dn;
  dn.m = M;
  dn.n = mid;
  dn.k = p.down->kp;
  dn.out = h->mid32;
  dn.ldo = mid;
  dn.row_scale = h->scales;
  dn.col_scale = p.down->scales;
  dn.status = h->status;
  dn.layer = layer;
  return gemm_launch(kGemmI8, kEpiResF32, h->q, p.down->q, dn, s);
}

// The nested forward; `trace` as documented for kb_forward_trace.
int forward_nested(kb_handle* h, int n, const float* d_spatial, const float* d_global, const int* d_sym, float* d_out,
                   uint16_t* trace) {
  kb_model* m = h->model;
  const kb_model_desc& d = m->desc;
  const int c = d.trunk_channels, mid = d.mid_channels, M = n * kSeq;
  cudaStream_t s = h->stream;
  const size_t plane = static_cast<size_t>(M) * c;
  const float scale = nested_attention_scale();
  int rc = stem_gather_launch(d_spatial, d_global, d_sym, h->stem_a, n, h->nhwc, s, 1);
  if (!rc) rc = f16_gemm_f32(h, h->stem_a, m->stem_w, M, c, kStemK, h->x32, nullptr);
  for (int bi = 0; bi < d.num_blocks && !rc; ++bi) {
    const NestedBlock& b = m->nblocks[bi];
    // pre_bn gate of the raw trunk (the stem's conv_bias_gate for block 0)
    rc = gate_silu_launch(h->x32, c, b.pre_s, b.pre_b, h->x, c, M, c, 1, s);
    if (!rc && trace)
      rc = check_cuda(cudaMemcpyAsync(trace + bi * plane, h->x, plane * 2, cudaMemcpyDeviceToDevice, s), "trace");
    if (!rc) rc = f16_gemm_f32(h, h->x, b.pre_w, M, mid, c, h->mid32, nullptr);
    for (size_t pi = 0; pi < b.pairs.size() && !rc; ++pi)
      rc = nested_pair(h, b.pairs[pi], static_cast<unsigned>(bi * d.pairs_per_block + pi), n, scale);
    // post_bn gate of the inner stream, then the mid -> C linear into the raw trunk
    if (!rc) rc = gate_silu_launch(h->mid32, mid, b.post_s, b.post_b, h->att, mid, M, mid, 1, s);
    if (!rc) rc = f16_gemm_f32(h, h->att, b.post_w, M, c, mid, h->x32, h->x32);
  }
  if (rc) return rc;
  rc = gate_silu_launch(h->x32, c, m->tip_gamma, m->tip_beta, h->att, c, M, c, 1, s);
  if (!rc && trace)
    for (int i = d.num_blocks; i < d.num_blocks + 2 && !rc; ++i)
      rc = check_cuda(cudaMemcpyAsync(trace + i * plane, h->att, plane * 2, cudaMemcpyDeviceToDevice, s), "trace");
  if (rc) return rc;
  {
    GemmArgs g;
    g.m = M;
    g.n = kHeadN;
    g.k = c;
    g.out = h->hp;
    g.ldo = kHeadN;
    g.bias = m->head_b;
    g.ab_f16 = 1;
    rc = gemm_launch(kGemmBF16, kEpiF32, h->att, m->head_w, g, s);
    if (rc) return rc;
  }
  float* pol = d_out;
  float* val = pol + static_cast<size_t>(n) * 6 * 362;
  float* misc = val + static_cast<size_t>(n) * 3;
  float* more = misc + static_cast<size_t>(n) * 10;
  float* own = more + static_cast<size_t>(n) * 8;
  return heads_launch(h->hp, m->head_ptrs, pol, val, misc, more, own, n, h->status, s);
}

// One forward pass of n positions on device buffers, enqueued on `s`.  When
// `trace` is non-null it receives bf16 [(num_blocks + 2), n*361, C]: the stem
// output, each block's attention output, and the final residual stream.
int forward(kb_handle* h, int n, const float* d_spatial, const float* d_global, const int* d_sym, float* d_out,
            uint16_t* trace = nullptr) {
  kb_model* m = h->model;
  const kb_model_desc& d = m->desc;
  const int c = d.trunk_channels, f = d.ffn_channels, M = n * kSeq;
  cudaStream_t s = h->stream;
  int rc = check_cuda(cudaMemsetAsync(h->status, 0, sizeof(unsigned), s), "status reset");
  if (!rc) rc = check_cuda(cudaMemsetAsync(h->status + 1, 0xff, sizeof(unsigned), s), "status reset");
  if (rc) return rc;
  if (d.topology == KB_TOPO_NESTED) return forward_nested(h, n, d_spatial, d_global, d_sym, d_out, trace);
  rc = stem_gather_launch(d_spatial, d_global, d_sym, h->stem_a, n, h->nhwc, s);
  if (rc) return rc;
  {
    GemmArgs g;
    g.m = M;
    g.n = c;
    g.k = kStemK;
    g.out = h->x;
    g.ldo = c;
    g.out_f16 = 0;
    rc = gemm_launch(kGemmBF16, kEpi16, h->stem_a, m->stem_w, g, s);
    if (rc) return rc;
  }
  const size_t plane = static_cast<size_t>(M) * c;
  if (trace) {
    rc = check_cuda(cudaMemcpyAsync(trace, h->x, plane * 2, cudaMemcpyDeviceToDevice, s), "trace copy");
    if (rc) return rc;
  }
  const float scale = 1.0f / sqrtf(static_cast<float>(d.head_dim));
  for (int bi = 0; bi < d.num_blocks; ++bi) {
    const Block& b = m->blocks[bi];
    const unsigned layer = static_cast<unsigned>(bi);
    if (m->mixed) {
      rc = mixed_block(h, b, layer, n, scale, trace ? trace + (1 + bi) * plane : nullptr);
      if (rc) return rc;
      continue;
    }
    if (d.precision == KB_PREC_MXFP8) {
      rc = mxfp8_block(h, b, layer, n, scale, trace ? trace + (1 + bi) * plane : nullptr);
      if (rc) return rc;
      continue;
    }
    // attention
    rc = quantize_rows_launch(h->x, KB_DT_BF16, c, M, c, b.qkv->kp, true, b.rms1, m->eps, 0, h->q, h->scales,
                              h->status, layer, s);
    if (rc) return rc;
    GemmArgs g;
    g.m = M;
    g.n = 3 * c;
    g.k = b.qkv->kp;
    g.out = h->qkv;
    g.ldo = 3 * c;
    g.row_scale = h->scales;
    g.col_scale = b.qkv->scales;
    g.out_f16 = 0;
    g.status = h->status;
    g.layer = layer;
    set_rope(g, b, d);
    rc = gemm_launch(kGemmI8, kEpiRope16, h->q, b.qkv->q, g, s);
    if (rc) return rc;
    rc = check_cuda(cudaMemsetAsync(h->row_amax, 0, static_cast<size_t>(M) * sizeof(uint32_t), s), "amax reset");
    if (rc) return rc;
    // Q and K were rotated by the QKV projection's epilogue: no tables here.
    rc = attention_launch(h->qkv, nullptr, nullptr, h->att, n, kSeq, d.num_heads, d.head_dim, scale, 0, s,
                          h->row_amax, h->status);
    if (rc) return rc;
    if (trace) {
      rc = check_cuda(cudaMemcpyAsync(trace + (1 + bi) * plane, h->att, plane * 2, cudaMemcpyDeviceToDevice, s),
                      "trace copy");
      if (rc) return rc;
    }
    rc = quantize_rows_amax_launch(h->att, KB_DT_BF16, c, h->row_amax, M, c, b.out->kp, h->q, h->scales,
                                   h->status, layer, s);
    if (rc) return rc;
    GemmArgs o;
    o.m = M;
    o.n = c;
    o.k = b.out->kp;
    o.out = h->x;
    o.ldo = c;
    o.row_scale = h->scales;
    o.col_scale = b.out->scales;
    o.out_f16 = 0;
    o.status = h->status;
    o.layer = layer;
    rc = gemm_launch(kGemmI8, kEpiRes16, h->q, b.out->q, o, s);
    if (rc) return rc;
    // FFN
    rc = quantize_rows_launch(h->x, KB_DT_BF16, c, M, c, b.up->kp, true, b.rms2, m->eps, 0, h->q, h->scales,
                              h->status, layer, s);
    if (rc) return rc;
    rc = check_cuda(cudaMemsetAsync(h->row_amax, 0, static_cast<size_t>(M) * sizeof(uint32_t), s), "amax reset");
    if (rc) return rc;
    GemmArgs u;
    u.row_amax = h->row_amax;
    u.m = M;
    u.n = f;
    u.k = b.up->kp;
    u.out = h->hidden;
    u.ldo = f;
    u.row_scale = h->scales;
    u.col_scale = b.up->scales;
    u.bias = b.up_b;
    u.act = 1;
    u.out_f16 = 0;
    u.status = h->status;
    u.layer = layer;
    rc = gemm_launch(kGemmI8, kEpi16, h->q, b.up->q, u, s);
    if (rc) return rc;
    rc = quantize_rows_amax_launch(h->hidden, KB_DT_BF16, f, h->row_amax, M, f, b.down->kp, h->q, h->scales,
                                   h->status, layer, s);
    if (rc) return rc;
    GemmArgs dn;
    dn.m = M;
    dn.n = c;
    dn.k = b.down->kp;
    dn.out = h->x;
    dn.ldo = c;
    dn.row_scale = h->scales;
    dn.col_scale = b.down->scales;
    dn.bias = b.down_b;
    dn.out_f16 = 0;
    dn.status = h->status;
    dn.layer = layer;
    rc = gemm_launch(kGemmI8, kEpiRes16, h->q, b.down->q, dn, s);
    if (rc) return rc;
  }
  if (trace) {
    rc = check_cuda(cudaMemcpyAsync(trace + (1 + d.num_blocks) * plane, h->x, plane * 2, cudaMemcpyDeviceToDevice, s),
                    "trace copy");
    if (rc) return rc;
  }
  rc = trunk_tip_launch(h->x, m->tip_gamma, m->tip_beta, h->att, M, c, s);
  if (rc) return rc;
  {
    GemmArgs g;
    g.m = M;
    g.n = kHeadN;
    g.k = c;
    g.out = h->hp;
    g.ldo = kHeadN;
    g.bias = m->head_b;
    rc = gemm_launch(kGemmBF16, kEpiF32, h->att, m->head_w, g, s);
    if (rc) return rc;
  }
  float* pol = d_out;
  float* val = pol + static_cast<size_t>(n) * 6 * 362;
  float* misc = val + static_cast<size_t>(n) * 3;
  float* more = misc + static_cast<size_t>(n) * 10;
  float* own = more + static_cast<size_t>(n) * 8;
  return heads_launch(h->hp, m->head_ptrs, pol, val, misc, more, own, n, h->status, s);
}

// Forward through a CUDA graph per batch size: the first call for a size runs
// directly (so lazy module loading and function attributes happen outside
// capture), the second captures and instantiates, later calls replay.
int run_forward(kb_handle* h, int n, const float* d_spatial, const float* d_global, const int* d_sym, float* d_out,
                bool use_graph) {
  if (!use_graph) return forward(h, n, d_spatial, d_global, d_sym, d_out);
  const kb_handle::GraphKey key{n, d_spatial, d_global, d_sym, d_out};
  auto it = h->graphs.find(key);
  if (it != h->graphs.end()) return check_cuda(cudaGraphLaunch(it->second, h->stream), "graph launch");
  if (!h->warmed[key]) {
    h->warmed[key] = 1;
    return forward(h, n, d_spatial, d_global, d_sym, d_out);
  }
  cudaGraph_t graph = nullptr;
  int rc = check_cuda(cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
  if (rc) return rc;
  const int frc = forward(h, n, d_spatial, d_global, d_sym, d_out);
  rc = check_cuda(cudaStreamEndCapture(h->stream, &graph), "end capture");
  if (frc) {
    if (graph) cudaGraphDestroy(graph);
    return frc;
  }
  if (rc) return rc;
  cudaGraphExec_t exec = nullptr;
  rc = check_cuda(cudaGraphInstantiate(&exec, graph, 0), "graph instantiate");
  cudaGraphDestroy(graph);
  if (rc) return rc;
  h->graphs[key] = exec;
  return check_cuda(cudaGraphLaunch(exec, h->stream), "graph launch");
}

void destroy_handle(kb_handle* h) {
  if (!h) return;
  for (auto& kv : h->graphs) cudaGraphExecDestroy(kv.second);
  for (auto& sl : h->slots) {
    cudaFreeHost(sl.h_spatial);
    cudaFreeHost(sl.h_global);
    cudaFreeHost(sl.h_out);
    cudaFreeHost(sl.h_status);
    cudaFree(sl.d_spatial);
    cudaFree(sl.d_global);
    cudaFree(sl.d_out);
    cudaFreeHost(sl.h_post);
    cudaFreeHost(sl.h_dec);
    cudaFree(sl.d_post);
    cudaFree(sl.d_dec);
    if (sl.done) cudaEventDestroy(sl.done);
    if (sl.inputs_ready) cudaEventDestroy(sl.inputs_ready);
  }
  cudaFree(h->stem_a);
  cudaFree(h->x);
  cudaFree(h->qkv);
  cudaFree(h->att);
  cudaFree(h->hidden);
  cudaFree(h->q);
  cudaFree(h->scales);
  cudaFree(h->mx_scales);
  cudaFree(h->row_amax);
  cudaFree(h->hp);
  cudaFree(h->x32);
  cudaFree(h->mid32);
  cudaFree(h->status);
  if (h->stream) cudaStreamDestroy(h->stream);
  if (h->copy_stream) cudaStreamDestroy(h->copy_stream);
  delete h;
}

// The nested blocks of the weight blob (layout in katab200.h): 16-bit weights
// as binary16, the SwiGLU FFN and the projections resolved to INT8 quantised
// per output channel (QuantizedWeights::new, int8.rs:171-211), the dual FFN
// weight [gate; up] tile-interleaved as kb_int8_weight_upload packs it.
int load_nested(kb_model* m, BlobCursor& cur) {
  const kb_model_desc& d = m->desc;
  const int c = d.trunk_channels, mid = d.mid_channels, hid = d.ffn_channels, nh = d.num_heads;
  m->nblocks.resize(d.num_blocks);
  int rc = KB_OK;
  for (int bi = 0; bi < d.num_blocks && !rc; ++bi) {
    NestedBlock& b = m->nblocks[bi];
    const float* pre_s = cur.take(c);
    const float* pre_b = cur.take(c);
    const float* pre_w = cur.take(static_cast<size_t>(mid) * c);
    rc = upload(&b.pre_s, pre_s, c, "upload gate");
    if (!rc) rc = upload(&b.pre_b, pre_b, c, "upload gate");
    if (!rc) rc = upload_f16(&b.pre_w, pre_w, static_cast<size_t>(mid) * c);
    b.pairs.resize(d.pairs_per_block);
    for (int pi = 0; pi < d.pairs_per_block && !rc; ++pi) {
      NestedPair& p = b.pairs[pi];
      const float* rms1 = cur.take(mid);
      const float* qkv = cur.take(3ull * mid * mid);
      const float* ow = cur.take(1ull * mid * mid);
      const float* freqs = cur.take(static_cast<size_t>(nh) * (kNestedHeadDim / 2) * 2);
      const float* rms2 = cur.take(mid);
      const float* gate = cur.take(1ull * hid * mid);
      const float* up = cur.take(1ull * hid * mid);
      const float* down = cur.take(1ull * mid * hid);
      rc = upload(&p.rms1, rms1, mid, "upload rms");
      if (!rc) rc = upload(&p.rms2, rms2, mid, "upload rms");
      if (!rc)
        rc = m->prec[KB_PROJ_QKV] == KB_PROJ_INT8 ? kb_int8_weight_upload(qkv, 3 * mid, mid, KB_LAYOUT_PLAIN, &p.qkv)
                                                  : upload_f16(&p.hqkv, qkv, 3ull * mid * mid);
      if (!rc)
        rc = m->prec[KB_PROJ_OUT] == KB_PROJ_INT8 ? kb_int8_weight_upload(ow, mid, mid, KB_LAYOUT_PLAIN, &p.out)
                                                  : upload_f16(&p.hout, ow, 1ull * mid * mid);
      if (!rc) {
        std::vector<float> dual(2ull * hid * mid);
        memcpy(dual.data(), gate, sizeof(float) * hid * mid);
        memcpy(dual.data() + static_cast<size_t>(hid) * mid, up, sizeof(float) * hid * mid);
        rc = kb_int8_weight_upload(dual.data(), 2 * hid, mid, KB_LAYOUT_SWIGLU_DUAL, &p.dual);
      }
      if (!rc) rc = kb_int8_weight_upload(down, mid, hid, KB_LAYOUT_PLAIN, &p.down);
      if (!rc) rc = upload_rope(freqs, nh, kNestedHeadDim, &p.rope_cos, &p.rope_sin);
    }
    if (rc) break;
    const float* post_s = cur.take(mid);
    const float* post_b = cur.take(mid);
    const float* post_w = cur.take(static_cast<size_t>(c) * mid);
    rc = upload(&b.post_s, post_s, mid, "upload gate");
    if (!rc) rc = upload(&b.post_b, post_b, mid, "upload gate");
    if (!rc) rc = upload_f16(&b.post_w, post_w, static_cast<size_t>(c) * mid);
  }
  return rc;
}

}  // namespace

extern "C" {

int kb_model_blob_floats(const kb_model_desc* desc, size_t* count) {
  int rc = validate_desc(desc);
  if (rc) return rc;
  if (!count) {
    set_error("null count");
    return KB_E_INVALID;
  }
  *count = blob_floats(*desc);
  return KB_OK;
}

int kb_model_load(const kb_model_desc* desc, const float* blob, size_t count, int device, kb_model** out) {
  if (!out) {
    set_error("null output handle");
    return KB_E_INVALID;
  }
  *out = nullptr;
  int rc = validate_desc(desc);
  if (rc) return rc;
  if (!blob || count != blob_floats(*desc)) {
    set_error("weight blob size mismatch (see kb_model_blob_floats)");
    return KB_E_INVALID;
  }
  for (size_t i = 0; i < count; ++i) {
    if (!std::isfinite(blob[i])) {
      set_error("model weights contain NaN or infinity");
      return KB_E_INVALID;
    }
  }
  rc = check_cuda(cudaSetDevice(device), "cudaSetDevice");
  if (rc) return rc;
  rc = kb_device_check(device);
  if (rc) return rc;
  kb_model* m = new (std::nothrow) kb_model;
  if (!m) {
    set_error("out of host memory");
    return KB_E_INVALID;
  }
  m->desc = *desc;
  m->device = device;
  const kb_model_desc& d = *desc;
  resolve_precision(d, m->prec);
  {
    const int base = d.precision == KB_PREC_MXFP8 ? KB_PROJ_MXFP8 : KB_PROJ_INT8;
    for (int i = 0; i < 4; ++i) m->mixed = m->mixed || m->prec[i] != base;
  }
  const int c = d.trunk_channels, f = d.ffn_channels, nh = d.num_heads, hd = d.head_dim;
  BlobCursor cur{blob, count};
  const bool nested = d.topology == KB_TOPO_NESTED;
  if (d.norm_eps > 0.0f) m->eps = d.norm_eps;
  // stem [C, 217] -> 16-bit [C, 224] (bf16 flat, binary16 nested)
  {
    const float* w = cur.take(static_cast<size_t>(c) * kStemKUsed);
    std::vector<uint16_t> wb(static_cast<size_t>(c) * kStemK, 0);
    for (int r = 0; r < c; ++r)
      for (int k = 0; k < kStemKUsed; ++k)
        wb[static_cast<size_t>(r) * kStemK + k] = bits16(w[r * kStemKUsed + k], nested);
    rc = upload(&m->stem_w, wb.data(), wb.size(), "upload stem");
  }
  if (nested && !rc) rc = load_nested(m, cur);
  m->blocks.resize(nested ? 0 : d.num_blocks);
  for (int bi = 0; bi < static_cast<int>(m->blocks.size()) && !rc; ++bi) {
    Block& b = m->blocks[bi];
    const float* rms1 = cur.take(c);
    const float* qkv = cur.take(3ull * c * c);
    const float* ow = cur.take(1ull * c * c);
    const float* rms2 = cur.take(c);
    const float* up = cur.take(1ull * f * c);
    const float* up_b = cur.take(f);
    const float* dn = cur.take(1ull * c * f);
    const float* dn_b = cur.take(c);
    const float* freqs = cur.take(static_cast<size_t>(nh) * (hd / 2) * 2);
    rc = upload(&b.rms1, rms1, c, "upload rms");
    if (!rc) rc = upload(&b.rms2, rms2, c, "upload rms");
    // Each projection in its resolved precision.
    const float* srcs[4] = {qkv, ow, up, dn};
    const int ns[4] = {3 * c, c, f, c}, ks[4] = {c, c, c, f};
    kb_int8_weight** i8[4] = {&b.qkv, &b.out, &b.up, &b.down};
    kb_mxfp8_weight** mx[4] = {&b.mqkv, &b.mout, &b.mup, &b.mdown};
    uint16_t** b16[4] = {&b.bqkv, &b.bout, &b.bup, &b.bdown};
    for (int pi = 0; pi < 4 && !rc; ++pi) {
      if (m->prec[pi] == KB_PROJ_INT8) {
        rc = kb_int8_weight_upload(srcs[pi], ns[pi], ks[pi], KB_LAYOUT_PLAIN, i8[pi]);
      } else if (m->prec[pi] == KB_PROJ_MXFP8) {
        rc = kb_mxfp8_weight_upload(srcs[pi], ns[pi], ks[pi], ks[pi], mx[pi]);
      } else {
        std::vector<uint16_t> wb(static_cast<size_t>(ns[pi]) * ks[pi]);
        for (size_t e = 0; e < wb.size(); ++e) wb[e] = bf16_bits(srcs[pi][e]);
        rc = upload(b16[pi], wb.data(), wb.size(), "upload bf16 projection");
      }
    }
    if (!rc) rc = upload(&b.up_b, up_b, f, "upload bias");
    if (!rc) rc = upload(&b.down_b, dn_b, c, "upload bias");
    if (!rc) rc = upload_rope(freqs, nh, hd, &b.rope_cos, &b.rope_sin);
  }
  if (!rc) {
    const float* tg = cur.take(c);
    const float* tb = cur.take(c);
    rc = upload(&m->tip_gamma, tg, c, "upload tip");
    if (!rc) rc = upload(&m->tip_beta, tb, c, "upload tip");
  }
  if (!rc) {
    const float* p1 = cur.take(96ull * c);
    const float* g1 = cur.take(96ull * c);
    const float* g1b = cur.take(96);
    const float* v1 = cur.take(192ull * c);
    const float* v1b = cur.take(192);
    std::vector<uint16_t> hw(static_cast<size_t>(kHeadN) * c);
    std::vector<float> hb(kHeadN, 0.0f);
    for (size_t i = 0; i < 96ull * c; ++i) {
      hw[i] = bits16(p1[i], nested);
      hw[96ull * c + i] = bits16(g1[i], nested);
    }
    for (size_t i = 0; i < 192ull * c; ++i) hw[192ull * c + i] = bits16(v1[i], nested);
    for (int i = 0; i < 96; ++i) hb[96 + i] = g1b[i];
    for (int i = 0; i < 192; ++i) hb[192 + i] = v1b[i];
    rc = upload(&m->head_w, hw.data(), hw.size(), "upload head linears");
    if (!rc) rc = upload(&m->head_b, hb.data(), hb.size(), "upload head bias");
    // small head weights, order = HeadWeights
    static const size_t sizes[15] = {96 * 288, 96 * 288, 96, 6 * 96, 96, 6 * 96, 192 * 576, 192,
                                     3 * 192,  3,        10 * 192, 10, 8 * 192, 8, 192};
    // blob order: g_matmul, pass1_w, pass1_b, pass2_w, bias2, conv2p_w, v2_w, v2_b,
    //             value_w, value_b, misc_w, misc_b, moremisc_w, moremisc_b, own_w
    size_t total = 0;
    for (size_t s : sizes) total += (s + 3) & ~static_cast<size_t>(3);
    std::vector<float> small(total, 0.0f);
    size_t off = 0;
    size_t offs[15];
    for (int i = 0; i < 15; ++i) {
      const float* src = cur.take(sizes[i]);
      memcpy(small.data() + off, src, sizes[i] * sizeof(float));
      offs[i] = off;
      off += (sizes[i] + 3) & ~static_cast<size_t>(3);
    }
    if (!rc) rc = upload(&m->small, small.data(), small.size(), "upload head weights");
    if (!rc)
      for (int i = 0; i < 15; ++i) m->head_ptrs[i] = m->small + offs[i];
  }
  if (!rc && cur.left != 0) {
    set_error("internal: weight blob not fully consumed");
    rc = KB_E_STATE;
  }
  if (rc) {
    destroy_model(m);
    return rc;
  }
  *out = m;
  return KB_OK;
}

void kb_model_destroy(kb_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  destroy_model(m);
}

int kb_handle_create(kb_model* model, int max_batch, int inputs_nhwc, kb_handle** out) {
  if (!out || !model || max_batch <= 0 || max_batch > 4096) {
    set_error("kb_handle_create: need a model and 1 <= max_batch <= 4096");
    return KB_E_INVALID;
  }
  *out = nullptr;
  int rc = check_cuda(cudaSetDevice(model->device), "cudaSetDevice");
  if (rc) return rc;
  kb_handle* h = new (std::nothrow) kb_handle;
  if (!h) {
    set_error("out of host memory");
    return KB_E_INVALID;
  }
  h->model = model;
  h->device = model->device;
  h->max_batch = max_batch;
  h->nhwc = inputs_nhwc ? 1 : 0;
  const kb_model_desc& d = model->desc;
  const size_t M = static_cast<size_t>(max_batch) * kSeq, c = d.trunk_channels, f = d.ffn_channels;
  size_t kq = c > f ? c : f;
  kq = (kq + 15) / 16 * 16;
  rc = check_cuda(cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking), "stream create");
  if (!rc) rc = check_cuda(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking), "stream create");
  if (!rc) rc = dev_alloc(&h->stem_a, M * kStemK, "workspace");
  if (!rc) rc = dev_alloc(&h->x, M * c, "workspace");
  if (!rc) rc = dev_alloc(&h->qkv, M * 3 * c, "workspace");
  if (!rc) rc = dev_alloc(&h->att, M * c, "workspace");
  if (!rc) rc = dev_alloc(&h->hidden, M * f, "workspace");
  if (!rc) rc = dev_alloc(&h->q, M * kq, "workspace");
  if (!rc) rc = dev_alloc(&h->scales, M, "workspace");
  bool any_mxfp8 = false;
  for (int i = 0; i < 4; ++i) any_mxfp8 = any_mxfp8 || model->prec[i] == KB_PROJ_MXFP8;
  if (!rc && any_mxfp8) {
    rc = mxfp8_dims(static_cast<long>(M), static_cast<long>(c > f ? c : f), nullptr, nullptr, nullptr,
                    &h->mx_scale_bytes);
    if (!rc) rc = dev_alloc(&h->mx_scales, h->mx_scale_bytes, "workspace");
    // Scale bytes of padding rows are never written by the quantisers: keep
    // them finite (zero) so they only ever scale zero-filled operand rows.
    if (!rc) rc = check_cuda(cudaMemset(h->mx_scales, 0, h->mx_scale_bytes), "workspace clear");
  }
  if (!rc) rc = dev_alloc(&h->row_amax, M, "workspace");
  if (!rc) rc = dev_alloc(&h->hp, M * kHeadN, "workspace");
  if (!rc && d.topology == KB_TOPO_NESTED) {
    rc = dev_alloc(&h->x32, M * c, "workspace");
    if (!rc) rc = dev_alloc(&h->mid32, M * static_cast<size_t>(d.mid_channels), "workspace");
  }
  if (!rc) rc = dev_alloc(&h->status, 2, "status word");
  for (auto& sl : h->slots) {
    const size_t ns = static_cast<size_t>(max_batch) * kInC * kSeq, ng = static_cast<size_t>(max_batch) * (kInG + 1),
                 no = static_cast<size_t>(max_batch) * kOutPerPos;
    if (!rc) rc = check_cuda(cudaMallocHost(&sl.h_spatial, ns * sizeof(float)), "pinned input");
    if (!rc) rc = check_cuda(cudaMallocHost(&sl.h_global, ng * sizeof(float)), "pinned input");
    if (!rc) rc = check_cuda(cudaMallocHost(&sl.h_out, no * sizeof(float)), "pinned output");
    if (!rc) rc = check_cuda(cudaMallocHost(&sl.h_status, 2 * sizeof(unsigned)), "pinned status");
    if (!rc) rc = dev_alloc(&sl.d_spatial, ns, "device input");
    if (!rc) rc = dev_alloc(&sl.d_global, ng, "device input");
    if (!rc) rc = dev_alloc(&sl.d_out, no, "device output");
    const size_t np = static_cast<size_t>(max_batch) * kPostPerPos, nd = static_cast<size_t>(max_batch) * kDecPerPos;
    if (!rc) rc = check_cuda(cudaMallocHost(&sl.h_post, np), "pinned row parameters");
    if (!rc) rc = check_cuda(cudaMallocHost(&sl.h_dec, nd * sizeof(float)), "pinned decoded output");
    if (!rc) rc = dev_alloc(&sl.d_post, np, "device row parameters");
    if (!rc) rc = dev_alloc(&sl.d_dec, nd, "device decoded output");
    if (!rc) rc = check_cuda(cudaEventCreateWithFlags(&sl.done, cudaEventDisableTiming), "event");
    if (!rc) rc = check_cuda(cudaEventCreateWithFlags(&sl.inputs_ready, cudaEventDisableTiming), "event");
  }
  if (rc) {
    destroy_handle(h);
    return rc;
  }
  *out = h;
  return KB_OK;
}

void kb_handle_destroy(kb_handle* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->copy_stream);
  cudaStreamSynchronize(h->stream);
  destroy_handle(h);
}

int kb_handle_stream(kb_handle* h, uintptr_t* stream) {
  if (!h || !stream) {
    set_error("null handle");
    return KB_E_INVALID;
  }
  *stream = reinterpret_cast<uintptr_t>(h->stream);
  return KB_OK;
}

int kb_forward_device(kb_handle* h, int n, const float* d_spatial, const float* d_global, float* d_out,
                      int use_graph) {
  if (!h || !d_spatial || !d_global || !d_out || n <= 0 || n > h->max_batch) {
    set_error("kb_forward_device: need 1 <= n <= max_batch and device buffers");
    return KB_E_INVALID;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  int rc = check_cuda(cudaSetDevice(h->device), "cudaSetDevice");
  if (rc) return rc;
  return run_forward(h, n, d_spatial, d_global, nullptr, d_out, use_graph != 0);
}

int kb_forward_trace(kb_handle* h, int n, const float* d_spatial, const float* d_global, float* d_out,
                     uint16_t* d_trace) {
  if (!h || !d_spatial || !d_global || !d_out || !d_trace || n <= 0 || n > h->max_batch) {
    set_error("kb_forward_trace: need 1 <= n <= max_batch and device buffers");
    return KB_E_INVALID;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  int rc = check_cuda(cudaSetDevice(h->device), "cudaSetDevice");
  if (rc) return rc;
  return forward(h, n, d_spatial, d_global, nullptr, d_out, d_trace);
}

int kb_read_status(kb_handle* h, uint32_t status[2]) {
  if (!h || !status) {
    set_error("null handle");
    return KB_E_INVALID;
  }
  int rc = check_cuda(cudaSetDevice(h->device), "cudaSetDevice");
  if (!rc) rc = check_cuda(cudaStreamSynchronize(h->stream), "stream sync");
  if (!rc) rc = check_cuda(cudaMemcpy(status, h->status, 2 * sizeof(unsigned), cudaMemcpyDeviceToHost), "status");
  return rc;
}

}  // extern "C"

namespace {

// kb_submit and kb_submit_rows: rows == nullptr returns the raw heads, else
// each row's symmetry comes from rows and the outputs are decoded on the
// device (post-processed when legal != nullptr) before the copy back.
int submit_impl(kb_handle* h, int n, const float* spatial, const float* global, const int* symmetry,
                const kb_row_params* rows, const uint8_t* legal, uint64_t* token) {
  if (!h || !spatial || !global || !token || n <= 0 || n > h->max_batch) {
    set_error("submit: need 1 <= n <= max_batch, host inputs and a token");
    return KB_E_INVALID;
  }
  if (rows) {
    const int rc = check_row_params(rows, n);
    if (rc) return rc;
  } else if (symmetry) {
    for (int i = 0; i < n; ++i)
      if (symmetry[i] < 0 || symmetry[i] > 7) {
        set_error("kb_submit: symmetry must be in 0..7");
        return KB_E_INVALID;
      }
  }
  std::lock_guard<std::mutex> lock(h->mu);
  int rc = check_cuda(cudaSetDevice(h->device), "cudaSetDevice");
  if (rc) return rc;
  Slot* sl = nullptr;
  for (auto& cand : h->slots)
    if (!cand.busy) {
      sl = &cand;
      break;
    }
  if (!sl) {
    set_error("both pipeline slots are in flight: finish one before submitting again");
    return KB_E_STATE;
  }
  const size_t ns = static_cast<size_t>(n) * kInC * kSeq, ng = static_cast<size_t>(n) * kInG;
  memcpy(sl->h_spatial, spatial, ns * sizeof(float));
  memcpy(sl->h_global, global, ng * sizeof(float));
  // The symmetries ride behind the global features: one copy carries both.
  int* h_sym = reinterpret_cast<int*>(sl->h_global + ng);
  if (rows)
    for (int i = 0; i < n; ++i) h_sym[i] = rows[i].symmetry;
  else if (symmetry)
    memcpy(h_sym, symmetry, static_cast<size_t>(n) * sizeof(int));
  else
    memset(h_sym, 0, static_cast<size_t>(n) * sizeof(int));
  const int* d_sym = reinterpret_cast<const int*>(sl->d_global + ng);
  cudaStream_t s = h->stream, cs = h->copy_stream;
  // The slot is free, so the forward that last read its device inputs has
  // completed (its `done` event was waited for): the copies may run now,
  // beside the other slot's forward, and the forward waits for them.
  rc = check_cuda(cudaMemcpyAsync(sl->d_spatial, sl->h_spatial, ns * sizeof(float), cudaMemcpyHostToDevice, cs), "H2D");
  if (!rc)
    rc = check_cuda(cudaMemcpyAsync(sl->d_global, sl->h_global, (ng + n) * sizeof(float), cudaMemcpyHostToDevice, cs),
                    "H2D");
  const size_t row_bytes = static_cast<size_t>(n) * sizeof(kb_row_params);
  if (!rc && rows) {
    // Row parameters, then the legality bytes: one copy.
    memcpy(sl->h_post, rows, row_bytes);
    if (legal) memcpy(sl->h_post + row_bytes, legal, static_cast<size_t>(n) * 362);
    rc = check_cuda(cudaMemcpyAsync(sl->d_post, sl->h_post, row_bytes + (legal ? static_cast<size_t>(n) * 362 : 0),
                                    cudaMemcpyHostToDevice, cs), "H2D");
  }
  if (!rc) rc = check_cuda(cudaEventRecord(sl->inputs_ready, cs), "event record");
  if (!rc) rc = check_cuda(cudaStreamWaitEvent(s, sl->inputs_ready, 0), "stream wait");
  if (!rc) rc = run_forward(h, n, sl->d_spatial, sl->d_global, d_sym, sl->d_out, true);
  if (rows) {
    if (!rc)
      rc = decode_rows_launch(n, sl->d_out, reinterpret_cast<const kb_row_params*>(sl->d_post),
                              legal ? sl->d_post + row_bytes : nullptr, h->pp, sl->d_dec, s);
    if (!rc)
      rc = check_cuda(cudaMemcpyAsync(sl->h_dec, sl->d_dec, static_cast<size_t>(n) * kDecPerPos * sizeof(float),
                                      cudaMemcpyDeviceToHost, s), "D2H");
  } else if (!rc) {
    rc = check_cuda(cudaMemcpyAsync(sl->h_out, sl->d_out, static_cast<size_t>(n) * kOutPerPos * sizeof(float),
                                    cudaMemcpyDeviceToHost, s), "D2H");
  }
  if (!rc)
    rc = check_cuda(cudaMemcpyAsync(sl->h_status, h->status, 2 * sizeof(unsigned), cudaMemcpyDeviceToHost, s), "D2H");
  if (!rc) rc = check_cuda(cudaEventRecord(sl->done, s), "event record");
  if (rc) return rc;
  sl->busy = true;
  sl->decoded = rows != nullptr;
  sl->n = n;
  sl->token = h->next_token++;
  *token = sl->token;
  return KB_OK;
}

// Wait for a token's slot and check its status word; on success *out is the
// slot (released) with its pinned outputs readable.
int finish_wait(kb_handle* h, uint64_t token, bool decoded, uint32_t status[2], Slot** out) {
  if (!h) {
    set_error("null handle");
    return KB_E_INVALID;
  }
  Slot* sl = nullptr;
  for (auto& cand : h->slots)
    if (cand.busy && cand.token == token) sl = &cand;
  if (!sl) {
    set_error("unknown or already finished token");
    return KB_E_STATE;
  }
  if (sl->decoded != decoded) {
    set_error(decoded ? "token was submitted by kb_submit: finish it with kb_finish"
                      : "token was submitted by kb_submit_rows: finish it with kb_finish_rows");
    return KB_E_STATE;
  }
  int rc = check_cuda(cudaEventSynchronize(sl->done), "event wait");
  sl->busy = false;
  if (rc) return rc;
  if (status) {
    status[0] = sl->h_status[0];
    status[1] = sl->h_status[1];
  }
  if (sl->h_status[0] != 0) {
    set_error("forward reported status flags " + std::to_string(sl->h_status[0]) + " at layer " +
              std::to_string(static_cast<int>(sl->h_status[1])) + "; outputs withheld");
    return KB_E_NONFINITE;
  }
  *out = sl;
  return KB_OK;
}

// Copy head-major blocks of `widths[i]` floats per row out of `src`.
void copy_heads(const float* src, int n, const int (&widths)[5], float* const (&dst)[5]) {
  for (int i = 0; i < 5; ++i) {
    const size_t cnt = static_cast<size_t>(n) * widths[i];
    if (dst[i]) memcpy(dst[i], src, cnt * sizeof(float));
    src += cnt;
  }
}

}  // namespace

extern "C" {

int kb_submit(kb_handle* h, int n, const float* spatial, const float* global, const int* symmetry,
              uint64_t* token) {
  return submit_impl(h, n, spatial, global, symmetry, nullptr, nullptr, token);
}

int kb_submit_rows(kb_handle* h, int n, const float* spatial, const float* global, const kb_row_params* rows,
                   const uint8_t* legal, uint64_t* token) {
  if (!rows) {
    set_error("kb_submit_rows: row parameters required");
    return KB_E_INVALID;
  }
  return submit_impl(h, n, spatial, global, nullptr, rows, legal, token);
}

int kb_set_postprocess(kb_handle* h, const kb_postprocess_params* pp) {
  if (!h || !pp) {
    set_error("kb_set_postprocess: null argument");
    return KB_E_INVALID;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  h->pp = *pp;
  return KB_OK;
}

int kb_query(kb_handle* h, uint64_t token) {
  if (!h) {
    set_error("null handle");
    return -KB_E_INVALID;
  }
  for (auto& sl : h->slots) {
    if (sl.busy && sl.token == token) {
      const cudaError_t e = cudaEventQuery(sl.done);
      if (e == cudaSuccess) return 1;
      if (e == cudaErrorNotReady) return 0;
      return -check_cuda(e, "event query");
    }
  }
  set_error("unknown or already finished token");
  return -KB_E_STATE;
}

int kb_finish(kb_handle* h, uint64_t token, float* policy, float* value, float* misc, float* moremisc,
              float* ownership, uint32_t status[2]) {
  Slot* sl = nullptr;
  const int rc = finish_wait(h, token, false, status, &sl);
  if (rc) return rc;
  copy_heads(sl->h_out, sl->n, {6 * 362, 3, 10, 8, kSeq}, {policy, value, misc, moremisc, ownership});
  return KB_OK;
}

int kb_finish_rows(kb_handle* h, uint64_t token, float* policy, float* value, float* misc, float* moremisc,
                   float* ownership, uint32_t status[2]) {
  Slot* sl = nullptr;
  const int rc = finish_wait(h, token, true, status, &sl);
  if (rc) return rc;
  copy_heads(sl->h_dec, sl->n, {362, 3, 4, 2, kSeq}, {policy, value, misc, moremisc, ownership});
  return KB_OK;
}

int kb_warmup(kb_handle* h, const int* batches, int count) {
  if (!h || (!batches && count > 0) || count < 0) {
    set_error("kb_warmup: invalid arguments");
    return KB_E_INVALID;
  }
  std::lock_guard<std::mutex> lock(h->mu);
  int rc = check_cuda(cudaSetDevice(h->device), "cudaSetDevice");
  for (int i = 0; i < count && !rc; ++i) {
    const int n = batches[i];
    if (n <= 0 || n > h->max_batch) {
      set_error("kb_warmup: batch size out of range");
      return KB_E_INVALID;
    }
    // Zero inputs (a fresh handle's device memory is not meaningful), then for
    // each pipeline slot one direct run and one captured run.
    for (auto& sl : h->slots) {
      if (!rc) rc = check_cuda(cudaMemsetAsync(sl.d_spatial, 0, static_cast<size_t>(n) * kInC * kSeq * sizeof(float), h->stream), "memset");
      if (!rc) rc = check_cuda(cudaMemsetAsync(sl.d_global, 0, static_cast<size_t>(n) * (kInG + 1) * sizeof(float), h->stream), "memset");
      const int* d_sym = reinterpret_cast<const int*>(sl.d_global + static_cast<size_t>(n) * kInG);
      for (int k = 0; k < 2 && !rc; ++k) rc = run_forward(h, n, sl.d_spatial, sl.d_global, d_sym, sl.d_out, true);
    }
  }
  if (!rc) rc = check_cuda(cudaStreamSynchronize(h->stream), "warmup sync");
  return rc;
}

}  // extern "C"

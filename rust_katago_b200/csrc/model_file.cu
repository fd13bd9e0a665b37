// Native KataGo model files of the reference's TF3 family -> the nested
// topology's descriptor and weight blob (host code).
//
// Reads the format the reference's parser reads (crates/kata_nn/src/
// model_parser.rs:35-1160): whitespace-separated text tokens for every name and
// scalar, weight arrays as text floats (.txt) or as "@BIN@" followed by raw
// little-endian fp32 (.bin), optionally gzip-compressed (.gz).  Only the graph
// the reference's native CUDA path runs is accepted (native_model.rs:21-165):
// model version 17, 22 spatial / 19 global inputs, no metadata encoder,
// standard trunk-tip BN, nested bottleneck blocks of attention / SwiGLU FFN
// pairs, D = 32 attention with learned 2-D RoPE, SiLU everywhere, unit BN
// scales in the heads.  Lowering follows native_model.rs:79-299: BN folded to
// scale / bias (model_parser.rs:249-298), matrices transposed to out-first,
// the two native policy channels mapped to rows 0 and 5 and the six score
// channels split into misc rows 0..3 and moremisc rows 0..1.
#include <math.h>
#include <stdio.h>
#include <string.h>
#include <zlib.h>

#include <cstdlib>
#include <new>
#include <string>
#include <vector>

#include "../../include/katab200.h"
#include "kb_internal.h"

using namespace kb;

namespace {

struct Fail {
  std::string msg;
};

[[noreturn]] void fail(const std::string& m) { throw Fail{"model file: " + m}; }

void require(bool ok, const std::string& m) {
  if (!ok) fail(m);
}

std::vector<char> read_file(const char* path) {
  FILE* f = fopen(path, "rb");
  if (!f) fail(std::string("cannot open ") + path);
  std::vector<char> buf;
  char chunk[1 << 16];
  size_t got;
  while ((got = fread(chunk, 1, sizeof(chunk), f)) > 0) buf.insert(buf.end(), chunk, chunk + got);
  const bool err = ferror(f) != 0;
  fclose(f);
  require(!err, std::string("read error on ") + path);
  return buf;
}

// gzip stream -> bytes; trailing bytes after the stream are an error
// (model_parser.rs:1148-1154).
std::vector<char> gunzip(const std::vector<char>& in) {
  z_stream zs;
  memset(&zs, 0, sizeof(zs));
  require(inflateInit2(&zs, 15 + 16) == Z_OK, "gzip init failed");
  zs.next_in = reinterpret_cast<Bytef*>(const_cast<char*>(in.data()));
  zs.avail_in = static_cast<uInt>(in.size());
  std::vector<char> out;
  char chunk[1 << 16];
  int rc;
  do {
    zs.next_out = reinterpret_cast<Bytef*>(chunk);
    zs.avail_out = sizeof(chunk);
    rc = inflate(&zs, Z_NO_FLUSH);
    if (rc != Z_OK && rc != Z_STREAM_END) {
      inflateEnd(&zs);
      fail("corrupt gzip data");
    }
    out.insert(out.end(), chunk, chunk + (sizeof(chunk) - zs.avail_out));
  } while (rc != Z_STREAM_END);
  const size_t left = zs.avail_in;
  inflateEnd(&zs);
  require(left == 0, "unexpected bytes after gzip model");
  return out;
}

bool space(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r' || c == '\f' || c == '\v'; }

struct Reader {
  const char* p;
  const char* end;
  bool binary;

  std::string token() {
    while (p < end && space(*p)) ++p;
    const char* s = p;
    while (p < end && !space(*p)) ++p;
    require(s != p, "unexpected end of file");
    return std::string(s, p);
  }
  int i32() {
    const std::string t = token();
    char* e = nullptr;
    const long v = strtol(t.c_str(), &e, 10);
    require(*e == 0 && v >= -2147483647L - 1 && v <= 2147483647L, "bad integer " + t);
    return static_cast<int>(v);
  }
  bool boolean() {
    const int v = i32();
    require(v == 0 || v == 1, "invalid boolean");
    return v == 1;
  }
  float f32() {
    const std::string t = token();
    char* e = nullptr;
    const float v = strtof(t.c_str(), &e);
    require(*e == 0 && std::isfinite(v), "bad or nonfinite float " + t);
    return v;
  }
  double f64() {
    const std::string t = token();
    char* e = nullptr;
    const double v = strtod(t.c_str(), &e);
    require(*e == 0 && std::isfinite(v), "bad or nonfinite scalar " + t);
    return v;
  }
  void reserved(int count, const char* what) {
    for (int i = 0; i < count; ++i) require(i32() == 0, std::string("unsupported ") + what + " option");
  }
  // A weight array of n floats: text tokens, or "@BIN@" then raw little-endian fp32.
  std::vector<float> floats(size_t n) {
    std::vector<float> v(n);
    if (!binary) {
      for (size_t i = 0; i < n; ++i) v[i] = f32();
      return v;
    }
    int before = 0;
    while (p < end && *p != '@') {
      require(space(*p), "non-whitespace before @BIN@ marker");
      ++p;
      require(++before <= 100, "could not find @BIN@ marker");
    }
    require(end - p >= 5 && memcmp(p, "@BIN@", 5) == 0, "expected @BIN@");
    p += 5;
    require(static_cast<size_t>(end - p) >= 4 * n, "truncated binary weight array");
    memcpy(v.data(), p, 4 * n);  // little-endian host
    p += 4 * n;
    for (float x : v) require(std::isfinite(x), "nonfinite binary weight");
    return v;
  }
};

size_t count_of(std::initializer_list<int> dims) {
  size_t n = 1;
  for (int d : dims) {
    require(d > 0 && d <= (1 << 20), "layer dimensions must be positive");
    n *= static_cast<size_t>(d);
    require(n <= (static_cast<size_t>(1) << 32), "layer dimensions overflow");
  }
  return n;
}

struct Conv {
  int ky = 0, kx = 0, ic = 0, oc = 0;
  std::vector<float> w;  // [oc, ic, ky, kx]
};
struct MatMul {
  int in = 0, out = 0;
  std::vector<float> w;  // as stored: [in, out]
  // out-first [out, in] (native_model.rs:375-388)
  std::vector<float> t() const {
    std::vector<float> r(w.size());
    for (int i = 0; i < in; ++i)
      for (int o = 0; o < out; ++o) r[static_cast<size_t>(o) * in + i] = w[static_cast<size_t>(i) * out + o];
    return r;
  }
};
struct BN {
  int c = 0;
  std::vector<float> scale, bias;  // merged affine
};

Conv conv(Reader& r) {
  r.token();  // name
  Conv c;
  c.ky = r.i32();
  c.kx = r.i32();
  c.ic = r.i32();
  c.oc = r.i32();
  const int dy = r.i32(), dx = r.i32();
  const size_t n = count_of({c.ky, c.kx, c.ic, c.oc});
  require(c.ky % 2 == 1 && c.kx % 2 == 1, "convolution filters must be odd");
  require(dy == 1 && dx == 1, "convolution dilation must be 1");
  const std::vector<float> src = r.floats(n);
  c.w.resize(n);
  // file: [Y, X, IC, OC] -> [OC, IC, Y, X] (model_parser.rs:219-234)
  for (int y = 0; y < c.ky; ++y)
    for (int x = 0; x < c.kx; ++x)
      for (int i = 0; i < c.ic; ++i)
        for (int o = 0; o < c.oc; ++o)
          c.w[((static_cast<size_t>(o) * c.ic + i) * c.ky + y) * c.kx + x] =
              src[((static_cast<size_t>(y) * c.kx + x) * c.ic + i) * c.oc + o];
  return c;
}

// Batch norm folded to merged scale / bias in fp32: scale / sqrt(var + eps),
// bias - scale' * mean (model_parser.rs:249-298).
BN bn(Reader& r) {
  r.token();
  BN b;
  b.c = r.i32();
  const float eps = r.f32();
  const bool has_scale = r.boolean(), has_bias = r.boolean();
  const size_t n = count_of({b.c});
  require(eps > 0.0f, "batch norm epsilon must be positive");
  const std::vector<float> mean = r.floats(n), var = r.floats(n);
  const std::vector<float> scale = has_scale ? r.floats(n) : std::vector<float>(n, 1.0f);
  const std::vector<float> bias = has_bias ? r.floats(n) : std::vector<float>(n, 0.0f);
  b.scale.resize(n);
  b.bias.resize(n);
  for (size_t i = 0; i < n; ++i) {
    const float ve = var[i] + eps;
    require(ve > 0.0f, "invalid batch norm variance");
    const float s = scale[i] / sqrtf(ve);
    const float sm = s * mean[i];
    const float bb = bias[i] - sm;
    require(std::isfinite(s) && std::isfinite(bb), "nonfinite merged batch norm affine");
    b.scale[i] = s;
    b.bias[i] = bb;
  }
  return b;
}

void silu_act(Reader& r) {
  r.token();
  const std::string kind = r.token();
  require(kind == "ACTIVATION_SILU", "native CUDA requires SiLU, got " + kind);
}

MatMul mm(Reader& r) {
  r.token();
  MatMul m;
  m.in = r.i32();
  m.out = r.i32();
  m.w = r.floats(count_of({m.in, m.out}));
  return m;
}

std::vector<float> mb(Reader& r, int channels) {
  r.token();
  const int c = r.i32();
  require(c == channels, "bias width mismatch");
  return r.floats(count_of({c}));
}

struct Rms {
  int c = 0;
  float eps = 0;
  std::vector<float> w;
};

Rms transformer_rms(Reader& r) {
  r.token();
  Rms n;
  n.c = r.i32();
  n.eps = r.f32();
  require(n.eps > 0.0f && n.eps <= 1.0f, "invalid transformer RMSNorm epsilon");
  n.w = r.floats(count_of({n.c}));
  return n;
}

struct Attention {
  Rms ln;
  MatMul q, k, v, o;
  std::vector<float> freqs;  // [heads, 16, 2]
};

Attention attention(Reader& r, int mid) {
  require(r.token() == "transformer_attention_block", "nested block must alternate attention then FFN");
  r.token();
  const int heads = r.i32(), kv = r.i32(), qd = r.i32(), vd = r.i32();
  const bool rope = r.boolean(), learnable = r.boolean();
  // native_model.rs:166-178: equal Q/K/V heads of width 32, learned 2-D RoPE
  require(qd == 32 && vd == 32 && heads == mid / 32 && kv == heads && rope && learnable,
          "native CUDA requires matching Q/K/V head counts, width 32 and learned 2D RoPE");
  Attention a;
  a.ln = transformer_rms(r);
  a.q = mm(r);
  a.k = mm(r);
  a.v = mm(r);
  a.o = mm(r);
  require(a.ln.c == mid && a.q.in == mid && a.k.in == mid && a.v.in == mid && a.q.out == mid && a.k.out == mid &&
              a.v.out == mid && a.o.in == mid && a.o.out == mid,
          "attention projection shapes");
  r.token();  // RoPE name
  const int rh = r.i32(), rp = r.i32(), last = r.i32();
  require(rh == heads && rp == 16 && last == 2, "native RoPE frequency shape must be [heads,16,2]");
  a.freqs = r.floats(count_of({heads, 16, 2}));
  return a;
}

struct Ffn {
  Rms ln;
  MatMul l1, gate, l2;
};

Ffn ffn(Reader& r, int mid, int* hidden) {
  require(r.token() == "transformer_ffn_block", "nested block must alternate attention then FFN");
  r.token();
  const int c = r.i32(), h = r.i32();
  const bool swiglu = r.boolean();
  require(c == mid && h > 0 && h <= 3 * mid && h % 8 == 0 && swiglu,
          "native CUDA requires SwiGLU FFN with matching mid channels and 8-aligned positive hidden width <= 3*mid");
  require(*hidden == 0 || *hidden == h, "every FFN of the model must have the same hidden width");
  *hidden = h;
  Ffn f;
  f.ln = transformer_rms(r);
  f.l1 = mm(r);
  f.gate = mm(r);
  f.l2 = mm(r);
  require(f.ln.c == mid && f.l1.in == mid && f.l1.out == h && f.gate.in == mid && f.gate.out == h &&
              f.l2.in == h && f.l2.out == mid,
          "FFN layer channel mismatch");
  return f;
}

void put(std::vector<float>& blob, const std::vector<float>& v) { blob.insert(blob.end(), v.begin(), v.end()); }

// rows `mapping` (from -> to) of a [rows_in, width] matrix into a zero [rows, width] one (native_model.rs:430-455)
std::vector<float> remap(const std::vector<float>& src, int width, int rows, std::initializer_list<std::pair<int, int>> m) {
  std::vector<float> out(static_cast<size_t>(rows) * width, 0.0f);
  for (const auto& ft : m)
    memcpy(out.data() + static_cast<size_t>(ft.second) * width, src.data() + static_cast<size_t>(ft.first) * width,
           sizeof(float) * width);
  return out;
}

struct Parsed {
  kb_model_desc desc;
  kb_postprocess_params pp;
  std::vector<float> blob;
};

Parsed parse_native(const char* path) {
  std::string lower(path);
  for (auto& ch : lower) ch = static_cast<char>(tolower(ch));
  auto ends = [&](const char* s) {
    const size_t n = strlen(s);
    return lower.size() >= n && lower.compare(lower.size() - n, n, s) == 0;
  };
  bool binary, compressed;
  if (ends(".bin.gz")) binary = true, compressed = true;
  else if (ends(".gz")) binary = false, compressed = true;
  else if (ends(".bin")) binary = true, compressed = false;
  else if (ends(".txt")) binary = false, compressed = false;
  else fail(std::string("unsupported model file extension: ") + path);
  std::vector<char> raw = read_file(path);
  if (compressed) raw = gunzip(raw);
  Reader r{raw.data(), raw.data() + raw.size(), binary};

  Parsed out;
  memset(&out.desc, 0, sizeof(out.desc));
  const std::string name = r.token();
  require(name.size() <= 96, "model name too long");
  const int version = r.i32();
  require(version == 17, "native CUDA requires model version 17");
  require(r.i32() == 22 && r.i32() == 19, "native CUDA requires 22 spatial / 19 global inputs");
  out.pp.model_version = version;
  out.pp.output_scale_multiplier = 1.0f;
  out.pp.td_score_multiplier = r.f64();
  out.pp.score_mean_multiplier = r.f64();
  out.pp.score_stdev_multiplier = r.f64();
  out.pp.lead_multiplier = r.f64();
  out.pp.variance_time_multiplier = r.f64();
  out.pp.shortterm_value_error_multiplier = r.f64();
  out.pp.shortterm_score_error_multiplier = r.f64();
  require(out.pp.td_score_multiplier > 0 && out.pp.score_mean_multiplier > 0 && out.pp.score_stdev_multiplier > 0 &&
              out.pp.lead_multiplier > 0 && out.pp.variance_time_multiplier > 0 &&
              out.pp.shortterm_value_error_multiplier > 0 && out.pp.shortterm_score_error_multiplier > 0,
          "postprocessing multipliers must be positive");
  require(r.i32() == 0, "native CUDA requires no metadata encoder");
  r.boolean();
  r.boolean();
  r.reserved(5, "model");

  // trunk (model_parser.rs:588-683)
  r.token();
  const int nb = r.i32(), c = r.i32(), mid = r.i32();
  r.i32();
  r.i32();
  r.i32();
  require(nb >= 1 && nb <= 64, "native CUDA requires 1..64 nested blocks");
  require(r.i32() == 0, "native CUDA requires standard trunk-tip BN");
  r.reserved(5, "trunk");
  const Conv stem = conv(r);
  const MatMul glob = mm(r);
  require(stem.ky == 3 && stem.kx == 3 && stem.ic == 22 && stem.oc == c && glob.in == 19 && glob.out == c,
          "initial convolution / matmul shapes");
  out.blob.reserve(64u << 20);
  // stem [C, 217]: the 3x3 taps (ic*9 + ky*3 + kx) then the 19 global weights
  {
    const std::vector<float> g = glob.t();
    for (int o = 0; o < c; ++o) {
      out.blob.insert(out.blob.end(), stem.w.begin() + static_cast<size_t>(o) * 198,
                      stem.w.begin() + static_cast<size_t>(o + 1) * 198);
      out.blob.insert(out.blob.end(), g.begin() + static_cast<size_t>(o) * 19, g.begin() + static_cast<size_t>(o + 1) * 19);
    }
  }
  int pairs = 0, hidden = 0;
  float eps = 0.0f;
  for (int b = 0; b < nb; ++b) {
    require(r.token() == "nested_bottleneck_block", "native CUDA requires only nested bottleneck trunk blocks");
    r.token();
    const int inner = r.i32();
    require(inner > 0 && inner % 2 == 0, "each native nested block must contain complete attention/FFN pairs");
    require(pairs == 0 || pairs == inner / 2, "every outer block must hold the same number of pairs");
    pairs = inner / 2;
    const BN pre = bn(r);
    silu_act(r);
    const Conv pre_conv = conv(r);
    require(pre.c == c && pre_conv.ky == 1 && pre_conv.ic == c && pre_conv.oc == mid, "nested pre_bn / pre_conv shapes");
    put(out.blob, pre.scale);
    put(out.blob, pre.bias);
    put(out.blob, pre_conv.w);
    for (int p = 0; p < pairs; ++p) {
      const Attention a = attention(r, mid);
      const Ffn f = ffn(r, mid, &hidden);
      require(eps == 0.0f || (eps == a.ln.eps && eps == f.ln.eps), "every RMSNorm must share one epsilon");
      eps = a.ln.eps;
      require(f.ln.eps == eps, "every RMSNorm must share one epsilon");
      put(out.blob, a.ln.w);
      put(out.blob, a.q.t());
      put(out.blob, a.k.t());
      put(out.blob, a.v.t());
      put(out.blob, a.o.t());
      put(out.blob, a.freqs);
      put(out.blob, f.ln.w);
      // C++ KataGo computes silu(linear1(x)) * linearGate(x) (native_model.rs:99-106)
      put(out.blob, f.l1.t());
      put(out.blob, f.gate.t());
      put(out.blob, f.l2.t());
    }
    const BN post = bn(r);
    silu_act(r);
    const Conv post_conv = conv(r);
    require(post.c == mid && post_conv.ky == 1 && post_conv.ic == mid && post_conv.oc == c,
            "nested post_bn / post_conv shapes");
    put(out.blob, post.scale);
    put(out.blob, post.bias);
    put(out.blob, post_conv.w);
  }
  const BN tip = bn(r);
  silu_act(r);
  require(tip.c == c, "trunk tip width");
  put(out.blob, tip.scale);
  put(out.blob, tip.bias);

  // policy head (model_parser.rs:685-740; native_model.rs:230-268)
  r.token();
  const int pc = r.i32();
  require(pc == 2 || pc == 4, "native v17 policy requires two or four output channels");
  r.reserved(3, "policy");
  const Conv p1 = conv(r), g1 = conv(r);
  const BN g1bn = bn(r);
  silu_act(r);
  const MatMul gbias = mm(r);
  const BN p1bn = bn(r);
  silu_act(r);
  const Conv p2 = conv(r);
  const MatMul pass1 = mm(r);
  const std::vector<float> pass1_b = mb(r, 96);
  silu_act(r);
  const MatMul pass2 = mm(r);
  require(p1.ky == 1 && p1.ic == c && p1.oc == 96 && g1.ky == 1 && g1.ic == c && g1.oc == 96 && g1bn.c == 96 &&
              p1bn.c == 96 && gbias.in == 288 && gbias.out == 96 && p2.ic == 96 && p2.oc == pc && pass1.in == 288 &&
              pass1.out == 96 && pass2.in == 96 && pass2.out == pc,
          "policy head shapes");
  for (int i = 0; i < 96; ++i)
    require(g1bn.scale[i] == 1.0f && p1bn.scale[i] == 1.0f,
            "native CUDA policy head requires unit BN scales");
  // value head (model_parser.rs:742-777; native_model.rs:270-299)
  r.token();
  r.reserved(3, "value");
  const Conv v1 = conv(r);
  const BN v1bn = bn(r);
  silu_act(r);
  const MatMul v2 = mm(r);
  const std::vector<float> v2_b = mb(r, 192);
  silu_act(r);
  const MatMul v3 = mm(r);
  const std::vector<float> v3_b = mb(r, 3);
  const MatMul sv3 = mm(r);
  const std::vector<float> sv3_b = mb(r, 6);
  const Conv own = conv(r);
  require(v1.ky == 1 && v1.ic == c && v1.oc == 192 && v1bn.c == 192 && v2.in == 576 && v2.out == 192 &&
              v3.in == 192 && v3.out == 3 && sv3.in == 192 && sv3.out == 6 && own.ic == 192 && own.oc == 1,
          "value head shapes (native CUDA requires value / score / ownership 3 / 6 / 1)");
  for (int i = 0; i < 192; ++i) require(v1bn.scale[i] == 1.0f, "native CUDA value head requires unit BN scales");
  while (r.p < r.end && space(*r.p)) ++r.p;
  require(r.p == r.end, "unexpected trailing model data");

  // heads in the blob order of kb_model_blob_floats (the BN scales are 1, so
  // the folded rows equal the convolutions)
  put(out.blob, p1.w);
  put(out.blob, g1.w);
  put(out.blob, g1bn.bias);
  put(out.blob, v1.w);
  put(out.blob, v1bn.bias);
  put(out.blob, gbias.t());
  put(out.blob, pass1.t());
  put(out.blob, pass1_b);
  put(out.blob, remap(pass2.t(), 96, 6, {{0, 0}, {1, 5}}));
  put(out.blob, p1bn.bias);
  put(out.blob, remap(p2.w, 96, 6, {{0, 0}, {1, 5}}));
  put(out.blob, v2.t());
  put(out.blob, v2_b);
  put(out.blob, v3.t());
  put(out.blob, v3_b);
  const std::vector<float> score = sv3.t();  // [6, 192]
  put(out.blob, remap(score, 192, 10, {{0, 0}, {1, 1}, {2, 2}, {3, 3}}));
  put(out.blob, remap(sv3_b, 1, 10, {{0, 0}, {1, 1}, {2, 2}, {3, 3}}));
  put(out.blob, remap(score, 192, 8, {{4, 0}, {5, 1}}));
  put(out.blob, remap(sv3_b, 1, 8, {{4, 0}, {5, 1}}));
  put(out.blob, own.w);

  kb_model_desc& d = out.desc;
  d.trunk_channels = c;
  d.num_blocks = nb;
  d.num_heads = mid / 32;
  d.head_dim = 32;
  d.ffn_channels = hidden;
  d.precision = KB_PREC_INT8;
  d.topology = KB_TOPO_NESTED;
  d.mid_channels = mid;
  d.pairs_per_block = pairs;
  d.norm_eps = eps;
  return out;
}

}  // namespace

extern "C" {

int kb_model_file_parse(const char* path, kb_model_desc* desc, float* blob, size_t capacity, size_t* count,
                        kb_postprocess_params* pp) {
  if (!path || !desc || !count) {
    set_error("kb_model_file_parse: path, desc and count are required");
    return KB_E_INVALID;
  }
  try {
    Parsed m = parse_native(path);
    size_t expect = 0;
    int rc = kb_model_blob_floats(&m.desc, &expect);
    if (rc) return rc;
    if (expect != m.blob.size()) {
      set_error("model file: parsed weights do not match the nested layout");
      return KB_E_INVALID;
    }
    *desc = m.desc;
    *count = m.blob.size();
    if (pp) *pp = m.pp;
    if (blob) {
      if (capacity < m.blob.size()) {
        set_error("kb_model_file_parse: blob capacity too small (see *count)");
        return KB_E_INVALID;
      }
      memcpy(blob, m.blob.data(), m.blob.size() * sizeof(float));
    }
    return KB_OK;
  } catch (const Fail& f) {
    set_error(f.msg);
    return KB_E_INVALID;
  } catch (const std::bad_alloc&) {
    set_error("model file: out of host memory");
    return KB_E_INVALID;
  }
}

int kb_model_load_file(const char* path, const kb_model_desc* recipe, int device, kb_model** out,
                       kb_postprocess_params* pp) {
  if (!out) {
    set_error("null output handle");
    return KB_E_INVALID;
  }
  *out = nullptr;
  try {
    Parsed m = parse_native(path ? path : "");
    if (recipe) {
      m.desc.precision = recipe->precision;
      memcpy(m.desc.proj_precision, recipe->proj_precision, sizeof(m.desc.proj_precision));
      m.desc.int8_min_ffn_width = recipe->int8_min_ffn_width;
    }
    if (pp) *pp = m.pp;
    return kb_model_load(&m.desc, m.blob.data(), m.blob.size(), device, out);
  } catch (const Fail& f) {
    set_error(f.msg);
    return KB_E_INVALID;
  } catch (const std::bad_alloc&) {
    set_error("model file: out of host memory");
    return KB_E_INVALID;
  }
}

}  // extern "C"

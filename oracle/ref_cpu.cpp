// ORACLE — test infrastructure only.  A CPU restatement of glypr's text-embedding path
// (crates/glypr-core, Rust + candle 0.11.0) used as the parity checker by tests/, by
// __graft_entry__.smoke() and as the timed CPU baseline in bench.py.  Nothing in the
// product (libglypr_cuda.so, glypr_b200/) links, loads or calls this file.
//
// Parity status: the reference cannot be compiled here (Rust/candle, no toolchain), so the
// model-level oracle is pinned only through the reference's own known-answer tests that
// touch the path (util.rs:258-306 MRL/L2, tests/test_cpu_simd.rs RMSNorm/GeGLU formula
// identity, the metal_kernels/mod.rs:1924-1979 Q8_0 GEMM recipe, corpus_parity.rs:420-494
// pooling precision).  End-to-end embeddings of the synthetic model are "parity unpinned"
// against the real reference; they are pinned against this restatement only.
//
// Followed line by line (paths relative to crates/glypr-core/src):
//   config.rs:76-250        metadata keys, layer pattern, per-layer head_dim / kv heads
//   model.rs:244-488        tensor names; token table dequantised to f32 (252-253)
//   model.rs:498-578        embed * sqrt(hidden), 24 layers, final norm + projection
//   model.rs:654-705        masked mean (f32), L2 (clamp 1e-12), MRL renormalise
//   layer.rs:20-50          pre-norm -> attn -> post-norm+res -> pre-FFN norm -> MLP -> post-norm+res
//   attention/mod.rs:95-277 q/k/v proj, per-head RMSNorm (v without weight), RoPE, repeat_kv
//   attention/standard.rs:61-82, chunked.rs:14-172  scores scale 1.0, softmax f32, window |i-j|<=W
//   norm.rs:22-94, cpu_simd/rmsnorm.rs:6-47   x * (1/sqrt(sum(x^2)/d + eps)) * w
//   rope.rs:14-106          inv_freq in f64 -> f32, freqs = pos * inv_freq (f32), NeoX halves
//   mlp.rs:31-70, cpu_simd/geglu.rs:6-18       tanh GELU with the +-10 clamp
//   linear.rs:150-172       Q8_0 linears through candle QMatMul on f32 activations
//   ple.rs:48-145, model.rs:257-275, 418-453, 527-542, layer.rs:44-49, norm.rs:65-94
//                           per-layer embeddings (when per_layer_model_proj.weight exists):
//                           P = RMSNorm_D(proj(x0) * f32(H^-0.5)) * w, [t, L, D]; after the FFN
//                           block h = (h + RMSNorm(proj_l(geglu(gate_l(h), P[:, l]))) * w_l) * s_l
// Third-party arithmetic restated from its published design (candle-core 0.11.0,
// Cargo.lock:258-261, not vendored): QMatMul on CPU quantises each activation row to Q8_0
// (ggml quantize_row_q8_0: d = amax/127, q = roundf(x/d)) and sums int8 block dot products
// scaled by f16(d_w) * f16(d_x) in f32 (vec_dot_q8_0_q8_0).  Mode M1 below.  Mode M2 is
// the exact f32 dequantisation f32(d)*q with f64 accumulation (the "fp32 dequantised
// reference" of the GEMM microbenchmark).
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fcntl.h>
#include <map>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <vector>
#include <immintrin.h>
#include <omp.h>

namespace {

// ------------------------------------------------------------------ fp16 / bf16 helpers
float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h >> 15) << 31;
  uint32_t exp = (h >> 10) & 0x1f;
  uint32_t man = h & 0x3ff;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {  // subnormal: renormalise
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400));
      man &= 0x3ff;
      bits = sign | (uint32_t)(127 - 15 - e) << 23 | man << 13;
    }
  } else if (exp == 31) {
    bits = sign | 0x7f800000u | man << 13;
  } else {
    bits = sign | (exp + 112) << 23 | man << 13;
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_f16(float f) {  // round to nearest even
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000;
  int32_t exp = (int32_t)((x >> 23) & 0xff) - 127 + 15;
  uint32_t man = x & 0x7fffff;
  if (((x >> 23) & 0xff) == 0xff) return (uint16_t)(sign | 0x7c00 | (man ? 0x200 : 0));
  if (exp >= 31) return (uint16_t)(sign | 0x7c00);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    man |= 0x800000;
    int shift = 14 - exp;
    uint32_t half = 1u << (shift - 1);
    uint32_t rem = man & ((1u << shift) - 1);
    uint32_t r = man >> shift;
    if (rem > half || (rem == half && (r & 1))) ++r;
    return (uint16_t)(sign | r);
  }
  uint32_t r = (uint32_t)exp << 10 | man >> 13;
  uint32_t rem = man & 0x1fff;
  if (rem > 0x1000 || (rem == 0x1000 && (r & 1))) ++r;
  return (uint16_t)(sign | r);
}

float bf16_to_f32(uint16_t b) {
  uint32_t bits = (uint32_t)b << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

// ------------------------------------------------------------------ GGUF (minimal reader)
enum { T_F32 = 0, T_F16 = 1, T_Q8_0 = 8, T_BF16 = 30 };

struct Tensor {
  std::vector<int64_t> ne;  // ne[0] innermost
  uint32_t type = 0;
  const uint8_t* data = nullptr;
  int64_t rows() const { return ne.size() > 1 ? ne[1] : 1; }
  int64_t cols() const { return ne[0]; }
};

struct Value {
  int type = -1;
  double num = 0;
  std::string str;
  std::vector<double> arr;
  int64_t arr_len = 0;
  int arr_type = -1;
};

struct Gguf {
  void* map = nullptr;
  size_t size = 0;
  std::map<std::string, Value> kv;
  std::map<std::string, Tensor> tensors;
  ~Gguf() {
    if (map) munmap(map, size);
  }
};

struct Reader {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <class T> T get() {
    T v{};
    if (p + sizeof(T) > end) { ok = false; return v; }
    memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    uint64_t n = get<uint64_t>();
    if (!ok || p + n > end) { ok = false; return {}; }
    std::string s((const char*)p, n);
    p += n;
    return s;
  }
};

bool read_scalar(Reader& r, int t, double* out, std::string* s) {
  switch (t) {
    case 0: *out = r.get<uint8_t>(); break;
    case 1: *out = r.get<int8_t>(); break;
    case 2: *out = r.get<uint16_t>(); break;
    case 3: *out = r.get<int16_t>(); break;
    case 4: *out = r.get<uint32_t>(); break;
    case 5: *out = r.get<int32_t>(); break;
    case 6: *out = r.get<float>(); break;
    case 7: *out = r.get<uint8_t>() ? 1 : 0; break;
    case 8: *s = r.str(); break;
    case 10: *out = (double)r.get<uint64_t>(); break;
    case 11: *out = (double)r.get<int64_t>(); break;
    case 12: *out = r.get<double>(); break;
    default: return false;
  }
  return r.ok;
}

bool gguf_open(const char* path, Gguf* g, std::string* err) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) { *err = std::string("cannot open ") + path; return false; }
  struct stat st;
  fstat(fd, &st);
  g->size = (size_t)st.st_size;
  g->map = mmap(nullptr, g->size, PROT_READ, MAP_PRIVATE, fd, 0);
  close(fd);
  if (g->map == MAP_FAILED) { g->map = nullptr; *err = "mmap failed"; return false; }
  Reader r{(const uint8_t*)g->map, (const uint8_t*)g->map + g->size};
  if (r.get<uint32_t>() != 0x46554747u) { *err = "not a GGUF file"; return false; }
  uint32_t version = r.get<uint32_t>();
  if (version < 2 || version > 3) { *err = "unsupported GGUF version"; return false; }
  uint64_t n_t = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
  for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
    std::string key = r.str();
    Value v;
    v.type = (int)r.get<uint32_t>();
    if (v.type == 9) {
      v.arr_type = (int)r.get<uint32_t>();
      v.arr_len = (int64_t)r.get<uint64_t>();
      for (int64_t j = 0; j < v.arr_len && r.ok; ++j) {
        double x = 0;
        std::string s;
        if (!read_scalar(r, v.arr_type, &x, &s)) { *err = "bad array"; return false; }
        if (v.arr_type != 8) v.arr.push_back(x);
      }
    } else if (!read_scalar(r, v.type, &v.num, &v.str)) {
      *err = "bad metadata value";
      return false;
    }
    g->kv[key] = v;
  }
  uint64_t align = 32;
  auto a = g->kv.find("general.alignment");
  if (a != g->kv.end()) align = (uint64_t)a->second.num;
  std::vector<std::pair<std::string, uint64_t>> offs;
  for (uint64_t i = 0; i < n_t && r.ok; ++i) {
    std::string name = r.str();
    Tensor t;
    uint32_t nd = r.get<uint32_t>();
    for (uint32_t d = 0; d < nd; ++d) t.ne.push_back((int64_t)r.get<uint64_t>());
    t.type = r.get<uint32_t>();
    offs.push_back({name, r.get<uint64_t>()});
    g->tensors[name] = t;
  }
  if (!r.ok) { *err = "truncated GGUF header"; return false; }
  size_t hdr = (size_t)(r.p - (const uint8_t*)g->map);
  size_t data0 = (hdr + align - 1) / align * align;
  for (auto& o : offs) {
    Tensor& t = g->tensors[o.first];
    int64_t n = 1;
    for (auto e : t.ne) n *= e;
    size_t bytes = t.type == T_F32 ? 4 * n : (t.type == T_F16 || t.type == T_BF16) ? 2 * n
                 : t.type == T_Q8_0 ? n / 32 * 34 : 0;
    if (!bytes || data0 + o.second + bytes > g->size) { *err = "tensor out of file: " + o.first; return false; }
    t.data = (const uint8_t*)g->map + data0 + o.second;
  }
  return true;
}

// ------------------------------------------------------------------ model
struct Linear {
  int64_t n = 0, k = 0;  // out, in
  uint32_t type = 0;
  const uint8_t* data = nullptr;
};

struct Layer {
  Linear q, k, v, o, gate, up, down;
  Linear ple_gate, ple_proj;  // PLE block (ple.rs:96-145): inp_gate [D, H], proj [H, D]
  std::vector<float> attn_norm, q_norm, k_norm, post_attn, ffn_norm, post_ffw, ple_post;
  float scalar = 1.0f;  // layer_output_scale (1 when absent)
  bool sliding = true;
  int head_dim = 256, n_kv = 1;
  double theta = 1e4;
};

}  // namespace

struct oracle_model {
  Gguf g;
  int n_layers = 0, hidden = 0, ffn = 0, n_heads = 0, vocab = 0, emb_out = 0, max_pos = 0;
  double eps = 1e-6;
  int window = 512;
  Tensor embd;
  std::vector<Layer> layers;
  std::vector<float> out_norm;
  std::vector<Linear> head;
  int ple_dim = 0;  // 0: no per-layer embeddings
  Linear ple_model_proj;
  std::vector<float> ple_norm;
  std::string err;
};

namespace {

thread_local std::string g_err;

double meta_num(const Gguf& g, const std::string& k, double dflt, bool* found = nullptr) {
  auto it = g.kv.find(k);
  if (found) *found = it != g.kv.end();
  return it == g.kv.end() ? dflt : it->second.num;
}

bool get_f32_vec(const Gguf& g, const std::string& name, int64_t n, std::vector<float>* out) {
  auto it = g.tensors.find(name);
  if (it == g.tensors.end()) { g_err = "missing tensor " + name; return false; }
  const Tensor& t = it->second;
  if (t.ne[0] != n) { g_err = "bad shape for " + name; return false; }
  out->resize(n);
  if (t.type == T_F32) memcpy(out->data(), t.data, 4 * n);
  else if (t.type == T_F16) for (int64_t i = 0; i < n; ++i) (*out)[i] = f16_to_f32(((const uint16_t*)t.data)[i]);
  else if (t.type == T_BF16) for (int64_t i = 0; i < n; ++i) (*out)[i] = bf16_to_f32(((const uint16_t*)t.data)[i]);
  else { g_err = "unsupported norm dtype for " + name; return false; }
  return true;
}

bool get_linear(const Gguf& g, const std::string& name, int64_t n, int64_t k, Linear* out) {
  auto it = g.tensors.find(name);
  if (it == g.tensors.end()) { g_err = "missing tensor " + name; return false; }
  const Tensor& t = it->second;
  if (t.ne.size() != 2 || t.ne[0] != k || t.ne[1] != n) { g_err = "bad shape for " + name; return false; }
  if (t.type != T_Q8_0 && t.type != T_BF16 && t.type != T_F32 && t.type != T_F16) { g_err = "unsupported dtype for " + name; return false; }
  *out = Linear{n, k, t.type, t.data};
  return true;
}

// Q8_0 block helpers -----------------------------------------------------------
inline float blk_d(const uint8_t* b) { uint16_t h; memcpy(&h, b, 2); return f16_to_f32(h); }

void dequant_row(const Linear& w, int64_t row, float* out) {
  if (w.type == T_Q8_0) {
    const uint8_t* r = w.data + row * (w.k / 32) * 34;
    for (int64_t b = 0; b < w.k / 32; ++b) {
      float d = blk_d(r + 34 * b);
      const int8_t* q = (const int8_t*)(r + 34 * b + 2);
      for (int j = 0; j < 32; ++j) out[32 * b + j] = (float)q[j] * d;
    }
  } else if (w.type == T_BF16) {
    const uint16_t* r = (const uint16_t*)w.data + row * w.k;
    for (int64_t j = 0; j < w.k; ++j) out[j] = bf16_to_f32(r[j]);
  } else if (w.type == T_F16) {
    const uint16_t* r = (const uint16_t*)w.data + row * w.k;
    for (int64_t j = 0; j < w.k; ++j) out[j] = f16_to_f32(r[j]);
  } else {
    memcpy(out, (const float*)w.data + row * w.k, 4 * w.k);
  }
}

struct QBlock { uint16_t d; int8_t qs[32]; };

// ggml quantize_row_q8_0: d = amax/127 (f32), id = 1/d, q = roundf(x*id); d stored as fp16.
void quantize_row_q8_0(const float* x, int64_t k, QBlock* y) {
  for (int64_t b = 0; b < k / 32; ++b) {
    const float* xs = x + 32 * b;
    float amax = 0.f;
    for (int j = 0; j < 32; ++j) amax = std::fmax(amax, std::fabs(xs[j]));
    float d = amax / 127.0f;
    float id = d != 0.f ? 1.0f / d : 0.f;
    y[b].d = f32_to_f16(d);
    for (int j = 0; j < 32; ++j) y[b].qs[j] = (int8_t)roundf(xs[j] * id);
  }
}

// SIMD switch for the CPU-baseline speed (oracle_set_simd): the vector paths below compute
// every value exactly as the scalar loops do (integer block dots are exact; each float
// accumulation keeps its order), which a test checks bit for bit.
bool g_simd = true;

#if defined(__AVX2__)
// Four int8 block dots (32 products each) of one activation block against four weight
// blocks: exact int32 sums [w0.x, w1.x, w2.x, w3.x].  |w| as unsigned bytes times x with w's
// sign (maddubs: pairs of products, at most 2 * 128 * 127 < 2^15), then pairs of int16 summed
// into int32 (madd with ones) and the lanes folded.  Activations never hold -128 (quantised
// to [-127, 127]), so negating them cannot overflow.
inline __m128i dot32x4(const int8_t* x, const int8_t* w0, const int8_t* w1, const int8_t* w2, const int8_t* w3) {
  const __m256i vx = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(x));
  const __m256i ones = _mm256_set1_epi16(1);
  auto one = [&](const int8_t* w) {
    const __m256i vw = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(w));
    const __m256i p16 = _mm256_maddubs_epi16(_mm256_sign_epi8(vw, vw), _mm256_sign_epi8(vx, vw));
    return _mm256_madd_epi16(p16, ones);
  };
  const __m256i a = one(w0), b = one(w1), c = one(w2), d = one(w3);
  const __m256i h = _mm256_hadd_epi32(_mm256_hadd_epi32(a, b), _mm256_hadd_epi32(c, d));
  return _mm_add_epi32(_mm256_castsi256_si128(h), _mm256_extracti128_si256(h, 1));
}
#endif

#if defined(__AVX2__)
// M1 with AVX2 block dots.  The scalar loop's float steps are a multiply, a multiply and an add
// per block (the compiler fuses none of them there); fp-contract=off keeps this function from
// fusing the vector multiply and add, so both paths round identically.
__attribute__((optimize("fp-contract=off"))) void linear_m1_avx2(const Linear& w, const std::vector<QBlock>& xq,
                                                                 int64_t m, float* y) {
  const int64_t n = w.n, k = w.k, nb = k / 32;
  (void)k;
  // scales converted once: weights [n][nb] transposed to [nb][n], activations [m][nb]
  std::vector<float> dw((size_t)(nb * n)), dx((size_t)(m * nb));
#pragma omp parallel for schedule(static)
  for (int64_t c = 0; c < n; ++c)
    for (int64_t b = 0; b < nb; ++b) dw[(size_t)(b * n + c)] = blk_d(w.data + (c * nb + b) * 34);
  for (int64_t i = 0; i < m * nb; ++i) dx[(size_t)i] = f16_to_f32(xq[(size_t)i].d);
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t c0 = 0; c0 < n; c0 += 4) {
    const uint8_t* wr = w.data + c0 * nb * 34;
    const int64_t rs = nb * 34;
    for (int64_t i = 0; i < m; ++i) {
      const QBlock* xr = &xq[(size_t)(i * nb)];
      __m128 sum = _mm_setzero_ps();
      for (int64_t b = 0; b < nb; ++b) {
        const int8_t* q0 = (const int8_t*)(wr + 34 * b + 2);
        const __m128 s = _mm_cvtepi32_ps(dot32x4(xr[b].qs, q0, q0 + rs, q0 + 2 * rs, q0 + 3 * rs));
        // sumf += (float)s * d_w * d_x, per column in block order, as the scalar loop
        sum = _mm_add_ps(sum, _mm_mul_ps(_mm_mul_ps(s, _mm_loadu_ps(&dw[(size_t)(b * n + c0)])),
                                         _mm_set1_ps(dx[(size_t)(i * nb + b)])));
      }
      float o[4];
      _mm_storeu_ps(o, sum);
      for (int j = 0; j < 4; ++j) y[i * n + c0 + j] = o[j];
    }
  }
}
#endif

// Y[M,N] = X[M,K] * W[N,K]^T.  mode 1 = candle-faithful (Q8_0 activations), 2 = exact f32 dequant.
void linear_forward(const Linear& w, const float* x, int64_t m, float* y, int mode) {
  const int64_t n = w.n, k = w.k, nb = k / 32;
  if (w.type == T_Q8_0 && mode == 1) {
    std::vector<QBlock> xq((size_t)(m * nb));
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < m; ++i) quantize_row_q8_0(x + i * k, k, &xq[(size_t)(i * nb)]);
#if defined(__AVX2__)
    if (g_simd && n % 4 == 0) {
      linear_m1_avx2(w, xq, m, y);
      return;
    }
#endif
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t c = 0; c < n; ++c) {
      const uint8_t* wr = w.data + c * nb * 34;
      for (int64_t i = 0; i < m; ++i) {
        const QBlock* xr = &xq[(size_t)(i * nb)];
        float sumf = 0.f;
        for (int64_t b = 0; b < nb; ++b) {
          const int8_t* qw = (const int8_t*)(wr + 34 * b + 2);
          int32_t s = 0;
          for (int j = 0; j < 32; ++j) s += (int32_t)qw[j] * (int32_t)xr[b].qs[j];
          sumf += (float)s * blk_d(wr + 34 * b) * f16_to_f32(xr[b].d);
        }
        y[i * n + c] = sumf;
      }
    }
    return;
  }
  // f32 weights (exact dequant for Q8_0; bf16/f16/f32 linears are Standard f32 linears in
  // the reference, linear.rs:48-54) with f64 accumulation.
#pragma omp parallel
  {
    std::vector<float> wrow((size_t)k);
#pragma omp for schedule(dynamic, 16)
    for (int64_t c = 0; c < n; ++c) {
      dequant_row(w, c, wrow.data());
      for (int64_t i = 0; i < m; ++i) {
        const float* xr = x + i * k;
        double acc = 0.0;
        for (int64_t j = 0; j < k; ++j) acc += (double)xr[j] * (double)wrow[j];
        y[i * n + c] = (float)acc;
      }
    }
  }
}

// cpu_simd/rmsnorm.rs:6-47 -- sum of squares, inv = 1/sqrt(sum/d + eps), out = x*inv*w
void rmsnorm_rows(const float* x, const float* w, int64_t rows, int64_t d, float eps, float* out) {
#pragma omp parallel for schedule(static) if (rows > 64)
  for (int64_t r = 0; r < rows; ++r) {
    const float* xr = x + r * d;
    float ss = 0.f;
    for (int64_t j = 0; j < d; ++j) ss = std::fma(xr[j], xr[j], ss);
    float inv = 1.0f / std::sqrt(ss / (float)d + eps);
    float* o = out + r * d;
    if (w) for (int64_t j = 0; j < d; ++j) o[j] = xr[j] * inv * w[j];
    else for (int64_t j = 0; j < d; ++j) o[j] = xr[j] * inv;
  }
}

// cpu_simd/geglu.rs:6-18
inline float geglu1(float g, float u) {
  if (g <= -10.0f) return 0.0f;
  if (g >= 10.0f) return g * u;
  float g3 = g * g * g;
  float inner = 0.7978846f * (g + 0.044715f * g3);
  float act = 0.5f * g * (1.0f + std::tanh(inner));
  return act * u;
}

// rope.rs:14-87: inv_freq_i = f32(1/theta^(2i/d)) (f64), freqs = f32(pos)*inv_freq (f32),
// emb = cat(freqs, freqs); tables are cos/sin of emb in f32.
void rope_tables(int d, double theta, int64_t s, float* cos_t, float* sin_t) {
  int half = d / 2;
  std::vector<float> inv(half);
  for (int i = 0; i < half; ++i) inv[i] = (float)(1.0 / std::pow(theta, (double)(2 * i) / (double)d));
#pragma omp parallel for schedule(static) if (s > 64)
  for (int64_t p = 0; p < s; ++p)
    for (int i = 0; i < d; ++i) {
      float f = (float)p * inv[i % half];
      cos_t[p * d + i] = std::cos(f);
      sin_t[p * d + i] = std::sin(f);
    }
}

// rope.rs:90-106: x*cos + rotate_half(x)*sin, rotate_half = cat(-x2, x1)
void apply_rope(float* x, int d, const float* c, const float* s) {
  int half = d / 2;
  std::vector<float> tmp(x, x + d);
  for (int i = 0; i < d; ++i) {
    float rot = i < half ? -tmp[i + half] : tmp[i - half];
    x[i] = tmp[i] * c[i] + rot * s[i];
  }
}

// One sequence's attention over T valid tokens. q [T, H*D], k/v [T, KV*D] (token-major,
// already normed + roped); out [T, H*D].  Scores scale 1.0; keys with |i-j| > W masked on
// sliding layers (model.rs:634-638, chunked.rs:14-50); softmax in f32 (max-subtracted).
void attention_seq(const float* q, const float* k, const float* v, int64_t t, int h, int kvh,
                   int d, int window, bool sliding, float* out) {
  const int rep = h / kvh;
#if defined(__AVX2__)
  if (g_simd && d % 32 == 0) {
    // The same arithmetic with the keys transposed per KV head (kt[kv][e][j]): eight keys'
    // scores advance together, each still one fma chain over e in order; o[e] for eight e at
    // a time, each still one fma chain over j in order.
    std::vector<float> kt((size_t)(kvh * d * t));
#pragma omp parallel for schedule(static)
    for (int64_t j = 0; j < t; ++j)
      for (int kv = 0; kv < kvh; ++kv)
        for (int e = 0; e < d; ++e) kt[((size_t)kv * d + e) * t + j] = k[(j * kvh + kv) * d + e];
#pragma omp parallel
    {
      std::vector<float> sc((size_t)t + 8);
#pragma omp for collapse(2) schedule(dynamic, 8)
      for (int hh = 0; hh < h; ++hh)
        for (int64_t i = 0; i < t; ++i) {
          const int kv = hh / rep;
          const float* qi = q + i * h * d + hh * d;
          const float* kk = kt.data() + (size_t)kv * d * t;
          int64_t j0 = 0, j1 = t;
          if (sliding) {
            j0 = i - window > 0 ? i - window : 0;
            j1 = i + window + 1 < t ? i + window + 1 : t;
          }
          int64_t j = j0;
          for (; j + 32 <= j1; j += 32) {  // four independent chains hide the fma latency
            __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
            for (int e = 0; e < d; ++e) {
              const __m256 qe = _mm256_set1_ps(qi[e]);
              const float* ke = kk + (size_t)e * t + j;
              a0 = _mm256_fmadd_ps(qe, _mm256_loadu_ps(ke), a0);
              a1 = _mm256_fmadd_ps(qe, _mm256_loadu_ps(ke + 8), a1);
              a2 = _mm256_fmadd_ps(qe, _mm256_loadu_ps(ke + 16), a2);
              a3 = _mm256_fmadd_ps(qe, _mm256_loadu_ps(ke + 24), a3);
            }
            _mm256_storeu_ps(&sc[(size_t)j], a0);
            _mm256_storeu_ps(&sc[(size_t)j + 8], a1);
            _mm256_storeu_ps(&sc[(size_t)j + 16], a2);
            _mm256_storeu_ps(&sc[(size_t)j + 24], a3);
          }
          for (; j + 8 <= j1; j += 8) {
            __m256 acc = _mm256_setzero_ps();
            for (int e = 0; e < d; ++e)
              acc = _mm256_fmadd_ps(_mm256_set1_ps(qi[e]), _mm256_loadu_ps(kk + (size_t)e * t + j), acc);
            _mm256_storeu_ps(&sc[(size_t)j], acc);
          }
          for (; j < j1; ++j) {
            float s = 0.f;
            for (int e = 0; e < d; ++e) s = std::fma(qi[e], kk[(size_t)e * t + j], s);
            sc[(size_t)j] = s;
          }
          float mx = -INFINITY;
          for (j = j0; j < j1; ++j) mx = std::fmax(mx, sc[(size_t)j]);
          float sum = 0.f;
          for (j = j0; j < j1; ++j) { sc[(size_t)j] = std::exp(sc[(size_t)j] - mx); sum += sc[(size_t)j]; }
          float* o = out + i * h * d + hh * d;
          for (j = j0; j < j1; ++j) sc[(size_t)j] = sc[(size_t)j] / sum;  // p_j, as the scalar loop forms it
          for (int e = 0; e < d; e += 32) {  // four independent chains per pass
            __m256 a0 = _mm256_setzero_ps(), a1 = a0, a2 = a0, a3 = a0;
            for (j = j0; j < j1; ++j) {
              const __m256 pj = _mm256_set1_ps(sc[(size_t)j]);
              const float* vj = v + j * kvh * d + kv * d + e;
              a0 = _mm256_fmadd_ps(pj, _mm256_loadu_ps(vj), a0);
              a1 = _mm256_fmadd_ps(pj, _mm256_loadu_ps(vj + 8), a1);
              a2 = _mm256_fmadd_ps(pj, _mm256_loadu_ps(vj + 16), a2);
              a3 = _mm256_fmadd_ps(pj, _mm256_loadu_ps(vj + 24), a3);
            }
            _mm256_storeu_ps(o + e, a0);
            _mm256_storeu_ps(o + e + 8, a1);
            _mm256_storeu_ps(o + e + 16, a2);
            _mm256_storeu_ps(o + e + 24, a3);
          }
        }
    }
    return;
  }
#endif
#pragma omp parallel
  {
    std::vector<float> sc((size_t)t);
#pragma omp for collapse(2) schedule(dynamic, 8)
    for (int hh = 0; hh < h; ++hh)
      for (int64_t i = 0; i < t; ++i) {
        const int kv = hh / rep;
        const float* qi = q + i * h * d + hh * d;
        int64_t j0 = 0, j1 = t;
        if (sliding) {
          j0 = i - window > 0 ? i - window : 0;
          j1 = i + window + 1 < t ? i + window + 1 : t;
        }
        float mx = -INFINITY;
        for (int64_t j = j0; j < j1; ++j) {
          const float* kj = k + j * kvh * d + kv * d;
          float s = 0.f;
          for (int e = 0; e < d; ++e) s = std::fma(qi[e], kj[e], s);
          sc[j] = s;
          mx = std::fmax(mx, s);
        }
        float sum = 0.f;
        for (int64_t j = j0; j < j1; ++j) { sc[j] = std::exp(sc[j] - mx); sum += sc[j]; }
        float* o = out + i * h * d + hh * d;
        for (int e = 0; e < d; ++e) o[e] = 0.f;
        for (int64_t j = j0; j < j1; ++j) {
          float p = sc[j] / sum;
          const float* vj = v + j * kvh * d + kv * d;
          for (int e = 0; e < d; ++e) o[e] = std::fma(p, vj[e], o[e]);
        }
      }
  }
}

bool load_model(oracle_model* m, const char* path) {
  std::string err;
  if (!gguf_open(path, &m->g, &err)) { g_err = err; return false; }
  const Gguf& g = m->g;
  const std::string a = "gemma-embedding2.";
  bool f;
  m->n_layers = (int)meta_num(g, a + "block_count", 0, &f);
  if (!f) { g_err = "Missing gemma-embedding2.block_count"; return false; }
  m->hidden = (int)meta_num(g, a + "embedding_length", 0, &f);
  if (!f) { g_err = "Missing gemma-embedding2.embedding_length"; return false; }
  m->ffn = (int)meta_num(g, a + "feed_forward_length", 0, &f);
  if (!f) { g_err = "Missing gemma-embedding2.feed_forward_length"; return false; }
  m->n_heads = (int)meta_num(g, a + "attention.head_count", 0, &f);
  if (!f) { g_err = "Missing gemma-embedding2.attention.head_count"; return false; }
  int hd_swa = (int)meta_num(g, a + "attention.key_length_swa", 256);
  int hd_full = (int)meta_num(g, a + "attention.key_length", 512);
  m->emb_out = (int)meta_num(g, a + "embedding_length_out", 768);
  m->max_pos = (int)meta_num(g, a + "context_length", 262144);
  m->eps = meta_num(g, a + "attention.layer_norm_rms_epsilon", 1e-6);
  double th_swa = meta_num(g, a + "rope.freq_base_swa", 10000.0);
  double th_full = meta_num(g, a + "rope.freq_base", 1000000.0);
  auto tok = g.kv.find("tokenizer.ggml.tokens");
  m->vocab = tok != g.kv.end() && tok->second.type == 9 ? (int)tok->second.arr_len : 262144;
  std::vector<bool> sliding(m->n_layers);
  auto pat = g.kv.find(a + "attention.sliding_window_pattern");
  for (int i = 0; i < m->n_layers; ++i) {
    if (pat != g.kv.end() && pat->second.type == 9) {
      if (i >= (int)pat->second.arr.size()) { g_err = "sliding_window_pattern too short"; return false; }
      sliding[i] = pat->second.arr[i] != 0;
    } else {
      sliding[i] = (i + 1) % 6 != 0;
    }
  }
  auto kvarr = g.kv.find(a + "attention.head_count_kv");
  int kv0 = kvarr != g.kv.end() && !kvarr->second.arr.empty() ? (int)kvarr->second.arr[0] : 2;
  auto te = g.tensors.find("token_embd.weight");
  if (te == g.tensors.end()) { g_err = "missing tensor token_embd.weight"; return false; }
  m->embd = te->second;
  if (m->embd.ne[0] != m->hidden) { g_err = "bad shape for token_embd.weight"; return false; }
  m->layers.resize(m->n_layers);
  const int64_t H = m->hidden;
  for (int i = 0; i < m->n_layers; ++i) {
    Layer& L = m->layers[i];
    std::string p = "blk." + std::to_string(i) + ".";
    L.sliding = sliding[i];
    L.head_dim = L.sliding ? hd_swa : hd_full;
    L.n_kv = kv0;
    if (!L.sliding) {
      L.n_kv = kvarr != g.kv.end() && i < (int)kvarr->second.arr.size() ? (int)kvarr->second.arr[i] : 1;
    }
    L.theta = L.sliding ? th_swa : th_full;
    const int64_t D = L.head_dim;
    if (!get_f32_vec(g, p + "attn_norm.weight", H, &L.attn_norm) ||
        !get_f32_vec(g, p + "post_attention_norm.weight", H, &L.post_attn) ||
        !get_f32_vec(g, p + "ffn_norm.weight", H, &L.ffn_norm) ||
        !get_f32_vec(g, p + "post_ffw_norm.weight", H, &L.post_ffw) ||
        !get_f32_vec(g, p + "attn_q_norm.weight", D, &L.q_norm) ||
        !get_f32_vec(g, p + "attn_k_norm.weight", D, &L.k_norm) ||
        !get_linear(g, p + "attn_q.weight", m->n_heads * D, H, &L.q) ||
        !get_linear(g, p + "attn_k.weight", L.n_kv * D, H, &L.k) ||
        !get_linear(g, p + "attn_v.weight", L.n_kv * D, H, &L.v) ||
        !get_linear(g, p + "attn_output.weight", H, m->n_heads * D, &L.o) ||
        !get_linear(g, p + "ffn_gate.weight", m->ffn, H, &L.gate) ||
        !get_linear(g, p + "ffn_up.weight", m->ffn, H, &L.up) ||
        !get_linear(g, p + "ffn_down.weight", H, m->ffn, &L.down))
      return false;
    auto sc = g.tensors.find(p + "layer_output_scale.weight");
    if (sc != g.tensors.end()) {
      std::vector<float> v;
      if (!get_f32_vec(g, sc->first, 1, &v)) return false;
      L.scalar = v[0];
    }
  }
  // model.rs:257-275 (TextPLE) and 418-440 (TextPLEBlock per layer)
  if (g.tensors.count("per_layer_model_proj.weight")) {
    m->ple_dim = (int)meta_num(g, a + "embedding_length_per_layer_input", 512);
    const int64_t D = m->ple_dim;
    if (!get_linear(g, "per_layer_model_proj.weight", m->n_layers * D, H, &m->ple_model_proj) ||
        !get_f32_vec(g, "per_layer_proj_norm.weight", D, &m->ple_norm))
      return false;
    for (int i = 0; i < m->n_layers; ++i) {
      Layer& L = m->layers[i];
      std::string p = "blk." + std::to_string(i) + ".";
      if (!get_linear(g, p + "inp_gate.weight", D, H, &L.ple_gate) ||
          !get_linear(g, p + "proj.weight", H, D, &L.ple_proj) ||
          !get_f32_vec(g, p + "post_norm.weight", H, &L.ple_post))
        return false;
      if (!g.tensors.count(p + "layer_output_scale.weight")) {
        g_err = "missing tensor " + p + "layer_output_scale.weight";
        return false;
      }
    }
  } else {
    for (int i = 0; i < m->n_layers; ++i) {
      std::string p = "blk." + std::to_string(i) + ".";
      if (g.tensors.count(p + "proj.weight") || g.tensors.count(p + "inp_gate.weight")) {
        g_err = "missing tensor per_layer_model_proj.weight";
        return false;
      }
    }
  }
  if (!get_f32_vec(g, "output_norm.weight", H, &m->out_norm)) return false;
  if (g.tensors.count("dense.0.weight")) {
    int64_t prev = H;
    for (int j = 0;; ++j) {
      auto it = g.tensors.find("dense." + std::to_string(j) + ".weight");
      if (it == g.tensors.end()) break;
      Linear l;
      if (!get_linear(g, it->first, it->second.ne[1], prev, &l)) return false;
      m->head.push_back(l);
      prev = l.n;
    }
  } else {
    auto it = g.tensors.find("output.weight");
    if (it == g.tensors.end()) { g_err = "missing tensor output.weight"; return false; }
    Linear l;
    if (!get_linear(g, "output.weight", it->second.ne[1], H, &l)) return false;
    m->head.push_back(l);
  }
  if (m->head.back().n != m->emb_out) { g_err = "head output dim != embedding_length_out"; return false; }
  return true;
}

// Forward of one sequence's valid tokens; writes per-token projected embeddings [t, emb_out].
// If stop_layer >= 0, writes the residual stream after that layer ([t, hidden]) instead.
void forward_seq(const oracle_model* m, const int32_t* ids, int64_t t, int mode, int stop_layer,
                 float* out) {
  const int64_t H = m->hidden;
  const float eps = (float)m->eps;
  std::vector<float> h((size_t)(t * H)), x((size_t)(t * H));
  // model.rs:507-508 -- Embedding over the f32-dequantised table, then * f32(sqrt(hidden))
  const float scale = (float)std::sqrt((double)H);
  Linear emb{m->embd.ne[1], m->embd.ne[0], m->embd.type, m->embd.data};
  for (int64_t i = 0; i < t; ++i) {
    dequant_row(emb, ids[i], &h[(size_t)(i * H)]);
    for (int64_t j = 0; j < H; ++j) h[(size_t)(i * H + j)] *= scale;
  }
  // ple.rs:48-93: P = RMSNorm(proj(x0) * f32(H^-0.5)) * w over each of the L slices of D
  const int64_t PD = m->ple_dim, NL = m->n_layers;
  std::vector<float> ple;
  if (PD) {
    ple.resize((size_t)(t * NL * PD));
    linear_forward(m->ple_model_proj, h.data(), t, ple.data(), mode);
    const float ps = (float)std::pow((double)H, -0.5);
    for (auto& v : ple) v *= ps;
    rmsnorm_rows(ple.data(), m->ple_norm.data(), t * NL, PD, eps, ple.data());
  }
  for (int l = 0; l < m->n_layers; ++l) {
    const Layer& L = m->layers[l];
    const int D = L.head_dim, NH = m->n_heads, KV = L.n_kv;
    rmsnorm_rows(h.data(), L.attn_norm.data(), t, H, eps, x.data());
    std::vector<float> q((size_t)(t * NH * D)), k((size_t)(t * KV * D)), v((size_t)(t * KV * D));
    linear_forward(L.q, x.data(), t, q.data(), mode);
    linear_forward(L.k, x.data(), t, k.data(), mode);
    linear_forward(L.v, x.data(), t, v.data(), mode);
    rmsnorm_rows(q.data(), L.q_norm.data(), t * NH, D, eps, q.data());
    rmsnorm_rows(k.data(), L.k_norm.data(), t * KV, D, eps, k.data());
    rmsnorm_rows(v.data(), nullptr, t * KV, D, eps, v.data());
    std::vector<float> ct((size_t)(t * D)), st((size_t)(t * D));
    rope_tables(D, L.theta, t, ct.data(), st.data());
    for (int64_t i = 0; i < t; ++i) {
      for (int hh = 0; hh < NH; ++hh) apply_rope(&q[(size_t)((i * NH + hh) * D)], D, &ct[(size_t)(i * D)], &st[(size_t)(i * D)]);
      for (int hh = 0; hh < KV; ++hh) apply_rope(&k[(size_t)((i * KV + hh) * D)], D, &ct[(size_t)(i * D)], &st[(size_t)(i * D)]);
    }
    std::vector<float> ctx((size_t)(t * NH * D)), y((size_t)(t * H));
    attention_seq(q.data(), k.data(), v.data(), t, NH, KV, D, m->window, L.sliding, ctx.data());
    linear_forward(L.o, ctx.data(), t, y.data(), mode);
    rmsnorm_rows(y.data(), L.post_attn.data(), t, H, eps, y.data());
    for (size_t i = 0; i < h.size(); ++i) h[i] += y[i];
    rmsnorm_rows(h.data(), L.ffn_norm.data(), t, H, eps, x.data());
    std::vector<float> gt((size_t)(t * m->ffn)), up((size_t)(t * m->ffn));
    linear_forward(L.gate, x.data(), t, gt.data(), mode);
    linear_forward(L.up, x.data(), t, up.data(), mode);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < gt.size(); ++i) gt[i] = geglu1(gt[i], up[i]);
    linear_forward(L.down, gt.data(), t, y.data(), mode);
    rmsnorm_rows(y.data(), L.post_ffw.data(), t, H, eps, y.data());
    if (PD) {
      for (size_t i = 0; i < h.size(); ++i) h[i] += y[i];
      // ple.rs:118-145: gate on the un-normalised residual, GeGLU with this layer's slice,
      // projection, post-norm, residual add, then the layer scalar (norm.rs:65-94)
      std::vector<float> pg((size_t)(t * PD));
      linear_forward(L.ple_gate, h.data(), t, pg.data(), mode);
      for (int64_t i = 0; i < t; ++i)
        for (int64_t j = 0; j < PD; ++j)
          pg[(size_t)(i * PD + j)] = geglu1(pg[(size_t)(i * PD + j)], ple[(size_t)((i * NL + l) * PD + j)]);
      linear_forward(L.ple_proj, pg.data(), t, y.data(), mode);
      rmsnorm_rows(y.data(), L.ple_post.data(), t, H, eps, y.data());
    }
    // without PLE the block is the identity and the layer scalar applies to the FFN sum
    for (size_t i = 0; i < h.size(); ++i) h[i] = (h[i] + y[i]) * L.scalar;
    if (l == stop_layer) {
      memcpy(out, h.data(), sizeof(float) * h.size());
      return;
    }
  }
  rmsnorm_rows(h.data(), m->out_norm.data(), t, H, eps, x.data());
  std::vector<float> cur = x;
  int64_t cd = H;
  for (const Linear& l : m->head) {
    std::vector<float> nxt((size_t)(t * l.n));
    linear_forward(l, cur.data(), t, nxt.data(), mode);
    cur.swap(nxt);
    cd = l.n;
  }
  memcpy(out, cur.data(), sizeof(float) * (size_t)(t * cd));
}

// model.rs:654-705: mean over valid tokens in f32 (count clamped to 1e-9), L2 normalise
// (norm clamped to 1e-12), optional MRL: first `dim` values renormalised.
void pool_normalize(const float* tok, int64_t t, int64_t e, int out_dim, float* out) {
  std::vector<float> pooled((size_t)e, 0.f);
  for (int64_t i = 0; i < t; ++i)
    for (int64_t j = 0; j < e; ++j) pooled[(size_t)j] += tok[i * e + j];
  float cnt = std::fmax((float)t, 1e-9f);
  for (auto& p : pooled) p /= cnt;
  float ss = 0.f;
  for (auto p : pooled) ss += p * p;
  float nrm = std::fmax(std::sqrt(ss), 1e-12f);
  for (auto& p : pooled) p /= nrm;
  if (out_dim < e) {
    float s2 = 0.f;
    for (int j = 0; j < out_dim; ++j) s2 += pooled[(size_t)j] * pooled[(size_t)j];
    float n2 = std::fmax(std::sqrt(s2), 1e-12f);
    for (int j = 0; j < out_dim; ++j) out[j] = pooled[(size_t)j] / n2;
  } else {
    for (int64_t j = 0; j < e; ++j) out[j] = pooled[(size_t)j];
  }
}

}  // namespace

extern "C" {

const char* oracle_last_error(void) { return g_err.c_str(); }

oracle_model* oracle_open(const char* path) {
  auto* m = new oracle_model();
  if (!load_model(m, path)) {
    delete m;
    return nullptr;
  }
  return m;
}

void oracle_close(oracle_model* m) { delete m; }

// out[0..9] = layers, hidden, ffn, heads, vocab, emb_out, max_pos, head_dim(layer0), kv(layer0), window
int oracle_info(const oracle_model* m, int* out) {
  out[0] = m->n_layers; out[1] = m->hidden; out[2] = m->ffn; out[3] = m->n_heads;
  out[4] = m->vocab; out[5] = m->emb_out; out[6] = m->max_pos;
  out[7] = m->n_layers ? m->layers[0].head_dim : 0;
  out[8] = m->n_layers ? m->layers[0].n_kv : 0;
  out[9] = m->window;
  return 0;
}

void oracle_set_threads(int n) { if (n > 0) omp_set_num_threads(n); }
void oracle_set_simd(int on) { g_simd = on != 0; }
int oracle_max_threads(void) { return omp_get_max_threads(); }

// ids [n_seq, max_len] right-padded; out [n_seq, out_dim] L2-normalised (MRL if out_dim < E).
int oracle_embed(const oracle_model* m, const int32_t* ids, const int32_t* lengths, int n_seq,
                 int max_len, int mode, int out_dim, float* out) {
  if (max_len > m->max_pos) {
    g_err = "Input sequence length (" + std::to_string(max_len) +
            ") exceeds model max_position_embeddings (" + std::to_string(m->max_pos) + ")";
    return 1;
  }
  if (out_dim <= 0 || out_dim > m->emb_out) { g_err = "bad out_dim"; return 1; }
  for (int s = 0; s < n_seq; ++s) {
    int64_t t = lengths[s];
    if (t < 0 || t > max_len) { g_err = "bad length"; return 1; }
    for (int64_t i = 0; i < t; ++i)
      if (ids[(int64_t)s * max_len + i] < 0 || ids[(int64_t)s * max_len + i] >= m->vocab) {
        g_err = "token id out of range";
        return 1;
      }
    if (t == 0) {
      for (int j = 0; j < out_dim; ++j) out[(int64_t)s * out_dim + j] = 0.f;
      continue;
    }
    std::vector<float> tok((size_t)(t * m->emb_out));
    forward_seq(m, ids + (int64_t)s * max_len, t, mode, -1, tok.data());
    pool_normalize(tok.data(), t, m->emb_out, out_dim, out + (int64_t)s * out_dim);
  }
  return 0;
}

// residual stream after `layer` for one sequence of t tokens: out [t, hidden]
int oracle_hidden(const oracle_model* m, const int32_t* ids, int t, int layer, int mode, float* out) {
  if (layer < 0 || layer >= m->n_layers) { g_err = "bad layer"; return 1; }
  forward_seq(m, ids, t, mode, layer, out);
  return 0;
}

// per-token projected embeddings (before pooling) for one sequence: out [t, emb_out]
int oracle_tokens(const oracle_model* m, const int32_t* ids, int t, int mode, float* out) {
  forward_seq(m, ids, t, mode, -1, out);
  return 0;
}

// ---- kernel-level restatements for unit tests --------------------------------------
void oracle_q8_0_dequant(const uint8_t* blocks, int64_t n_blocks, float* out) {
  for (int64_t b = 0; b < n_blocks; ++b) {
    float d = blk_d(blocks + 34 * b);
    const int8_t* q = (const int8_t*)(blocks + 34 * b + 2);
    for (int j = 0; j < 32; ++j) out[32 * b + j] = (float)q[j] * d;
  }
}

void oracle_q8_0_quantize(const float* x, int64_t n, uint8_t* blocks) {
  quantize_row_q8_0(x, n, (QBlock*)blocks);
}

int oracle_q8_0_matmul(const uint8_t* w, int n, int k, const float* x, int m, int mode, float* y) {
  if (k % 32) { g_err = "K must be a multiple of 32"; return 1; }
  Linear l{n, k, T_Q8_0, w};
  linear_forward(l, x, m, y, mode);
  return 0;
}

void oracle_rmsnorm(const float* x, const float* w, int64_t rows, int64_t d, float eps, float* out) {
  rmsnorm_rows(x, w, rows, d, eps, out);
}

void oracle_geglu(const float* g, const float* u, int64_t n, float* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = geglu1(g[i], u[i]);
}

void oracle_rope_tables(int d, double theta, int64_t s, float* c, float* sn) { rope_tables(d, theta, s, c, sn); }

void oracle_attention(const float* q, const float* k, const float* v, int64_t t, int h, int kvh,
                      int d, int window, int sliding, float* out) {
  attention_seq(q, k, v, t, h, kvh, d, window, sliding != 0, out);
}

void oracle_pool_normalize(const float* tok, int64_t t, int64_t e, int out_dim, float* out) {
  pool_normalize(tok, t, e, out_dim, out);
}

}  // extern "C"

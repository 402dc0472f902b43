// CPU forward of the Llama/Qwen2 decoder family over GGUF block weights (module fak_b200._cpu).
//
// Two roles:
//  * the CPU serving path (the "SmolLM2-135M Q8_0, 256 + 128 greedy on the CPU" configuration):
//    weights stay in their GGML blocks, activations are quantized to int8 per 32-block and every
//    inner product is an integer dot times the two block scales -- the scheme of the reference's
//    CPU Q8 path (internal/model/quant_forward.go, Go asm qdot8 kernels);
//  * an fp32 oracle (act_quant = false): weights are dequantized block by block and dotted with
//    fp32 activations, RoPE angles in float64, matching the reference cpu-ref backend
//    (internal/compute/cpuref.go:38-290).
// Rows of every matrix are split over a fixed pool of std::threads.  KV cache: contiguous fp32 per layer.
#include <torch/extension.h>

#include <cmath>
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include <algorithm>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>

namespace {

enum QT { F32 = 0, F16 = 1, Q8_0 = 8, Q4_K = 12, Q6_K = 14 };

// Persistent worker pool: parallel_for(n, fn) runs fn(begin, end) on contiguous slices.
class Pool {
 public:
  explicit Pool(int n) : n_(std::max(1, n)) {
    for (int i = 1; i < n_; i++) workers_.emplace_back([this, i] { loop(i); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
      gen_++;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int size() const { return n_; }
  void parallel_for(int64_t n, const std::function<void(int64_t, int64_t)>& fn) {
    if (n_ == 1 || n < 2) {
      fn(0, n);
      return;
    }
    std::unique_lock<std::mutex> g(mu_);
    fn_ = &fn;
    total_ = n;
    pending_ = n_ - 1;
    gen_++;
    g.unlock();
    cv_.notify_all();
    run_slice(0);
    g.lock();
    done_.wait(g, [this] { return pending_ == 0; });
    fn_ = nullptr;
  }

 private:
  void run_slice(int i) {
    const int64_t per = (total_ + n_ - 1) / n_;
    const int64_t b = std::min<int64_t>(total_, i * per), e = std::min<int64_t>(total_, b + per);
    if (b < e) (*fn_)(b, e);
  }
  void loop(int i) {
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> g(mu_);
      cv_.wait(g, [&] { return gen_ != seen; });
      seen = gen_;
      if (stop_) return;
      g.unlock();
      run_slice(i);
      g.lock();
      if (--pending_ == 0) done_.notify_one();
    }
  }
  int n_;
  std::vector<std::thread> workers_;
  std::mutex mu_;
  std::condition_variable cv_, done_;
  const std::function<void(int64_t, int64_t)>* fn_ = nullptr;
  int64_t total_ = 0;
  int pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
};

Pool& pool() {
  static Pool p((int)std::max(1u, std::thread::hardware_concurrency()));
  return p;
}

float h2f(uint16_t h) {
  const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 31, m = h & 1023;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = s << 31;
    } else {  // subnormal
      int ee = -1;
      uint32_t mm = m;
      do { ee++; mm <<= 1; } while ((mm & 1024) == 0);
      bits = (s << 31) | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 1023) << 13);
    }
  } else if (e == 31) {
    bits = (s << 31) | 0x7f800000u | (m << 13);
  } else {
    bits = (s << 31) | ((e + 112) << 23) | (m << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t rd16(const uint8_t* p) { return (uint16_t)p[0] | ((uint16_t)p[1] << 8); }

struct Mat {
  std::vector<uint8_t> raw;  // packed rows
  int qt = F32, rows = 0, cols = 0;
  int64_t row_bytes = 0;
};

int64_t row_bytes_of(int qt, int cols) {
  switch (qt) {
    case F32: return (int64_t)cols * 4;
    case F16: return (int64_t)cols * 2;
    case Q8_0: return (int64_t)cols / 32 * 34;
    case Q4_K: return (int64_t)cols / 256 * 144;
    case Q6_K: return (int64_t)cols / 256 * 210;
  }
  throw std::runtime_error("cpuref: unsupported block type " + std::to_string(qt));
}

// dequantize one row to fp32
void dequant_row(const Mat& m, int r, float* out) {
  const uint8_t* row = m.raw.data() + (int64_t)r * m.row_bytes;
  const int n = m.cols;
  if (m.qt == F32) {
    std::memcpy(out, row, (size_t)n * 4);
  } else if (m.qt == F16) {
    for (int i = 0; i < n; i++) out[i] = h2f(rd16(row + 2 * i));
  } else if (m.qt == Q8_0) {
    for (int b = 0; b < n / 32; b++) {
      const uint8_t* blk = row + b * 34;
      const float d = h2f(rd16(blk));
      for (int i = 0; i < 32; i++) out[b * 32 + i] = d * (float)(int8_t)blk[2 + i];
    }
  } else if (m.qt == Q4_K) {
    for (int sb = 0; sb < n / 256; sb++) {
      const uint8_t* blk = row + sb * 144;
      const float d = h2f(rd16(blk)), dmin = h2f(rd16(blk + 2));
      const uint8_t* s = blk + 4;
      for (int j = 0; j < 8; j++) {
        int sc, mn;
        if (j < 4) { sc = s[j] & 63; mn = s[j + 4] & 63; }
        else { sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4); mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
        const uint8_t* q = blk + 16 + (j / 2) * 32;
        const int sh = (j & 1) * 4;
        for (int l = 0; l < 32; l++) out[sb * 256 + j * 32 + l] = d * sc * ((q[l] >> sh) & 15) - dmin * mn;
      }
    }
  } else if (m.qt == Q6_K) {
    for (int sb = 0; sb < n / 256; sb++) {
      const uint8_t* blk = row + sb * 210;
      const float d = h2f(rd16(blk + 208));
      for (int e = 0; e < 256; e++) {
        const int hn = e / 128, k = (e % 128) / 32, l = e % 32;
        const int q = ((blk[hn * 64 + (k & 1) * 32 + l] >> ((k >> 1) * 4)) & 15) |
                      (((blk[128 + hn * 32 + l] >> (2 * k)) & 3) << 4);
        out[sb * 256 + e] = d * (float)(int8_t)blk[192 + e / 16] * (float)(q - 32);
      }
    }
  }
}

struct QAct {  // int8 activations per 32-block
  std::vector<int8_t> q;
  std::vector<float> d;
  void build(const float* x, int n) {
    q.resize(n);
    d.resize(n / 32);
    for (int b = 0; b < n / 32; b++) {
      float amax = 0.f;
      for (int i = 0; i < 32; i++) amax = std::max(amax, std::fabs(x[b * 32 + i]));
      const float s = amax / 127.f;
      d[b] = s;
      for (int i = 0; i < 32; i++) q[b * 32 + i] = (int8_t)(s > 0 ? std::nearbyint(x[b * 32 + i] / s) : 0);
    }
  }
};

// y[r] = W[r] . x  for all rows; Q8_0 rows take the integer path when act_quant
void matvec(const Mat& m, const float* x, const QAct* qa, float* y, bool act_quant) {
  const int R = m.rows, n = m.cols;
  if (act_quant && m.qt == Q8_0 && qa) {
    pool().parallel_for(R, [&](int64_t r0, int64_t r1) {
    for (int64_t r = r0; r < r1; r++) {
      const uint8_t* row = m.raw.data() + (int64_t)r * m.row_bytes;
      float acc = 0.f;
      for (int b = 0; b < n / 32; b++) {
        const uint8_t* blk = row + b * 34;
        const int8_t* wq = reinterpret_cast<const int8_t*>(blk + 2);
        const int8_t* xq = qa->q.data() + b * 32;
        int s = 0;
        for (int i = 0; i < 32; i++) s += (int)wq[i] * (int)xq[i];
        acc += h2f(rd16(blk)) * qa->d[b] * (float)s;
      }
      y[r] = acc;
    }
    });
    return;
  }
  pool().parallel_for(R, [&](int64_t r0, int64_t r1) {
    std::vector<float> w(n);
    for (int64_t r = r0; r < r1; r++) {
      dequant_row(m, (int)r, w.data());
      double acc = 0.0;
      for (int i = 0; i < n; i++) acc += (double)w[i] * (double)x[i];
      y[r] = (float)acc;
    }
  });
}

void rmsnorm(const float* x, const float* g, float eps, int n, float* y) {
  double ss = 0;
  for (int i = 0; i < n; i++) ss += (double)x[i] * x[i];
  const float inv = 1.f / std::sqrt((float)(ss / n) + eps);
  for (int i = 0; i < n; i++) y[i] = x[i] * inv * g[i];
}

struct Layer {
  std::vector<float> attn_norm, ffn_norm, qb, kb, vb, qn, kn;
  Mat q, k, v, o, gate, up, down;
};

}  // namespace

class CpuModel {
 public:
  CpuModel(py::dict cfg, bool act_quant) : act_quant_(act_quant) {
    L = cfg["n_layers"].cast<int>();
    d = cfg["d_model"].cast<int>();
    H = cfg["n_heads"].cast<int>();
    Hk = cfg["n_kv_heads"].cast<int>();
    D = cfg["head_dim"].cast<int>();
    F = cfg["ffn_dim"].cast<int>();
    V = cfg["vocab_size"].cast<int>();
    eps = cfg["rms_eps"].cast<float>();
    theta = cfg["rope_theta"].cast<double>();
    layers.resize(L);
  }

  void set_matrix(const std::string& name, int layer, int qt, int rows, int cols, py::bytes data) {
    Mat m;
    m.qt = qt;
    m.rows = rows;
    m.cols = cols;
    m.row_bytes = row_bytes_of(qt, cols);
    std::string s = data;
    if ((int64_t)s.size() != m.row_bytes * rows) throw std::runtime_error("cpuref: size mismatch for " + name);
    m.raw.assign(s.begin(), s.end());
    if (layer < 0) {
      if (name == "embed") embed = std::move(m);
      else if (name == "lm_head") lm_head = std::move(m);
      else throw std::runtime_error("cpuref: unknown matrix " + name);
      return;
    }
    Layer& Ly = layers.at(layer);
    if (name == "q") Ly.q = std::move(m);
    else if (name == "k") Ly.k = std::move(m);
    else if (name == "v") Ly.v = std::move(m);
    else if (name == "o") Ly.o = std::move(m);
    else if (name == "gate") Ly.gate = std::move(m);
    else if (name == "up") Ly.up = std::move(m);
    else if (name == "down") Ly.down = std::move(m);
    else throw std::runtime_error("cpuref: unknown matrix " + name);
  }

  void set_vector(const std::string& name, int layer, std::vector<float> v) {
    if (layer < 0) {
      if (name == "final_norm") final_norm = std::move(v);
      else throw std::runtime_error("cpuref: unknown vector " + name);
      return;
    }
    Layer& Ly = layers.at(layer);
    if (name == "attn_norm") Ly.attn_norm = std::move(v);
    else if (name == "ffn_norm") Ly.ffn_norm = std::move(v);
    else if (name == "q_bias") Ly.qb = std::move(v);
    else if (name == "k_bias") Ly.kb = std::move(v);
    else if (name == "v_bias") Ly.vb = std::move(v);
    else if (name == "q_norm") Ly.qn = std::move(v);
    else if (name == "k_norm") Ly.kn = std::move(v);
    else throw std::runtime_error("cpuref: unknown vector " + name);
  }

  void reset() {
    kcache.assign(L, {});
    vcache.assign(L, {});
    n_ctx = 0;
  }

  // feed one token at position n_ctx; returns logits
  std::vector<float> step(int token) {
    if (kcache.size() != (size_t)L) reset();
    std::vector<float> x(d), h(d), tmp(std::max({d, H * D, F, 2 * F}));
    dequant_row(embed, token, x.data());
    const int pos = n_ctx;
    std::vector<float> q(H * D), k(Hk * D), v(Hk * D), att(H * D), g(F), u(F);
    QAct qa;
    const int half = D / 2;
    std::vector<float> cs(half), sn(half);
    for (int j = 0; j < half; j++) {
      const double inv = 1.0 / std::pow(theta, (2.0 * j) / D);
      cs[j] = (float)std::cos(pos * inv);
      sn[j] = (float)std::sin(pos * inv);
    }
    auto rope = [&](float* vec, int heads) {
      for (int hh = 0; hh < heads; hh++) {
        float* p = vec + hh * D;
        for (int j = 0; j < half; j++) {
          const float a = p[j], b = p[j + half];
          p[j] = a * cs[j] - b * sn[j];
          p[j + half] = b * cs[j] + a * sn[j];
        }
      }
    };
    auto headnorm = [&](float* vec, int heads, const std::vector<float>& gw) {
      if (gw.empty()) return;
      for (int hh = 0; hh < heads; hh++) rmsnorm(vec + hh * D, gw.data(), eps, D, vec + hh * D);
    };
    for (int i = 0; i < L; i++) {
      Layer& Ly = layers[i];
      rmsnorm(x.data(), Ly.attn_norm.data(), eps, d, h.data());
      if (act_quant_) qa.build(h.data(), d);
      matvec(Ly.q, h.data(), &qa, q.data(), act_quant_);
      matvec(Ly.k, h.data(), &qa, k.data(), act_quant_);
      matvec(Ly.v, h.data(), &qa, v.data(), act_quant_);
      if (!Ly.qb.empty())
        for (int j = 0; j < H * D; j++) q[j] += Ly.qb[j];
      if (!Ly.kb.empty())
        for (int j = 0; j < Hk * D; j++) k[j] += Ly.kb[j];
      if (!Ly.vb.empty())
        for (int j = 0; j < Hk * D; j++) v[j] += Ly.vb[j];
      headnorm(q.data(), H, Ly.qn);
      headnorm(k.data(), Hk, Ly.kn);
      rope(q.data(), H);
      rope(k.data(), Hk);
      kcache[i].insert(kcache[i].end(), k.begin(), k.end());
      vcache[i].insert(vcache[i].end(), v.begin(), v.end());
      const int T = pos + 1, G = H / Hk;
      const float scale = 1.f / std::sqrt((float)D);
      pool().parallel_for(H, [&](int64_t h0, int64_t h1) {
      for (int64_t hh = h0; hh < h1; hh++) {
        const int kh = (int)hh / G;
        std::vector<float> s(T);
        float mx = -INFINITY;
        for (int t = 0; t < T; t++) {
          const float* kt = kcache[i].data() + ((int64_t)t * Hk + kh) * D;
          float acc = 0.f;
          for (int j = 0; j < D; j++) acc += q[hh * D + j] * kt[j];
          s[t] = acc * scale;
          mx = std::max(mx, s[t]);
        }
        double den = 0;
        for (int t = 0; t < T; t++) { s[t] = std::exp(s[t] - mx); den += s[t]; }
        for (int j = 0; j < D; j++) {
          double acc = 0;
          for (int t = 0; t < T; t++) acc += s[t] * vcache[i][((int64_t)t * Hk + kh) * D + j];
          att[hh * D + j] = (float)(acc / den);
        }
      }
      });
      if (act_quant_) qa.build(att.data(), H * D);
      matvec(Ly.o, att.data(), &qa, tmp.data(), act_quant_);
      for (int j = 0; j < d; j++) x[j] += tmp[j];
      rmsnorm(x.data(), Ly.ffn_norm.data(), eps, d, h.data());
      if (act_quant_) qa.build(h.data(), d);
      matvec(Ly.gate, h.data(), &qa, g.data(), act_quant_);
      matvec(Ly.up, h.data(), &qa, u.data(), act_quant_);
      for (int j = 0; j < F; j++) g[j] = g[j] / (1.f + std::exp(-g[j])) * u[j];
      if (act_quant_) qa.build(g.data(), F);
      matvec(Ly.down, g.data(), &qa, tmp.data(), act_quant_);
      for (int j = 0; j < d; j++) x[j] += tmp[j];
    }
    rmsnorm(x.data(), final_norm.data(), eps, d, h.data());
    if (act_quant_) qa.build(h.data(), d);
    std::vector<float> logits(V);
    matvec(lm_head, h.data(), &qa, logits.data(), act_quant_);
    n_ctx++;
    return logits;
  }

  std::vector<int> generate(std::vector<int> prompt, int n_new) {
    reset();
    std::vector<float> lg;
    for (int t : prompt) lg = step(t);
    std::vector<int> out;
    for (int i = 0; i < n_new; i++) {
      int best = 0;
      for (int j = 1; j < V; j++)
        if (lg[j] > lg[best]) best = j;
      out.push_back(best);
      if (i + 1 < n_new) lg = step(best);
    }
    return out;
  }

  int threads() const { return pool().size(); }

 private:
  bool act_quant_;
  int L, d, H, Hk, D, F, V;
  float eps;
  double theta;
  std::vector<Layer> layers;
  Mat embed, lm_head;
  std::vector<float> final_norm;
  std::vector<std::vector<float>> kcache, vcache;
  int n_ctx = 0;
};

// ---- MoE experts resident in host memory (CPU offload) -----------------------------------------
// The expert FFNs of a MoE layer run here while the dense projections, the router and attention
// stay on the GPU (the llama.cpp --n-cpu-moe split; reference: internal/model/moe_offload.go,
// splitKernel routing every expert weight to the host kernel).  A layer holds this rank's band of
// experts [e0, e0 + n): gate/up rows interleaved in blocks of 8 (the device layout: rows
// [16i, 16i+8) gate, [16i+8, 16i+16) up) and down rows, both in their GGML blocks.  ffn() adds
// sum_slot w[b, slot] * expert_{ids[b, slot]}(x[b]) to out[b] for the slots whose expert is in
// the band, the slots added in order so the result does not depend on the thread count.
class CpuExperts {
 public:
  CpuExperts(int64_t n_layers, int64_t d, int64_t f, int64_t gate, bool act_quant)
      : d_((int)d), f_((int)f), gate_((int)gate), act_quant_(act_quant), layers_(n_layers) {
    if (gate < 2 || gate > 4) throw std::runtime_error("CpuExperts: gate code 2 (SwiGLU), 3 (GeGLU) or 4 (OAI)");
  }

  void set_layer(int64_t layer, int64_t e0, int64_t n, torch::Tensor gate_up, int64_t qt_gu, torch::Tensor down,
                 int64_t qt_dn, c10::optional<torch::Tensor> bias_gu, c10::optional<torch::Tensor> bias_dn) {
    if (!(layer >= 0 && layer < (int64_t)layers_.size()))
      throw std::runtime_error("CpuExperts: layer");
    L& l = layers_[layer];
    l.e0 = (int)e0;
    l.n = (int)n;
    load(l.gu, gate_up, (int)qt_gu, (int)(n * 2 * f_), d_);
    load(l.dn, down, (int)qt_dn, (int)(n * d_), f_);
    l.bgu.clear();
    l.bdn.clear();
    if (bias_gu.has_value()) l.bgu = floats(*bias_gu, n * 2 * f_);
    if (bias_dn.has_value()) l.bdn = floats(*bias_dn, n * d_);
  }

  void ffn(int64_t layer, torch::Tensor x, torch::Tensor ids, torch::Tensor wts, torch::Tensor out) {
    if (!(layer >= 0 && layer < (int64_t)layers_.size() && layers_[layer].n > 0))
      throw std::runtime_error("CpuExperts: layer not set");
    const L& l = layers_[layer];
    if (!(!x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.dim() == 2 &&
                    x.size(1) == d_))
      throw std::runtime_error("CpuExperts: x [B, d] f32 on the host");
    const int B = (int)x.size(0);
    if (!(ids.scalar_type() == torch::kInt32 && ids.is_contiguous() && ids.dim() == 2 && ids.size(0) == B))
      throw std::runtime_error("CpuExperts: ids [B, k] int32");
    if (!(wts.scalar_type() == torch::kFloat32 && wts.is_contiguous() && wts.sizes() == ids.sizes()))
      throw std::runtime_error("CpuExperts: wts [B, k] f32");
    if (!(out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.sizes() == x.sizes()))
      throw std::runtime_error("CpuExperts: out [B, d] f32");
    const int k = (int)ids.size(1);
    const int* id = ids.data_ptr<int>();
    const float* w = wts.data_ptr<float>();
    const float* xp = x.data_ptr<float>();
    float* op = out.data_ptr<float>();
    py::gil_scoped_release nogil;
    std::vector<int> pb, pe;   // (token, local expert) of every slot routed into the band
    std::vector<float> pw;
    for (int b = 0; b < B; b++)
      for (int j = 0; j < k; j++) {
        const int e = id[b * k + j] - l.e0;
        if (e >= 0 && e < l.n) {
          pb.push_back(b);
          pe.push_back(e);
          pw.push_back(w[b * k + j]);
        }
      }
    const int P = (int)pb.size();
    if (P == 0) return;
    std::vector<QAct> qx(act_quant_ ? B : 0);
    for (int b = 0; b < (int)qx.size(); b++) qx[b].build(xp + (int64_t)b * d_, d_);
    // gate/up rows of every routed pair, then the gated product
    const int R = 2 * f_;
    std::vector<float> gu((size_t)P * R), h((size_t)P * f_), y((size_t)P * d_);
    pool().parallel_for((int64_t)P * R, [&](int64_t i0, int64_t i1) {
      std::vector<float> tmp(d_);
      for (int64_t i = i0; i < i1; i++) {
        const int p = (int)(i / R), r = (int)(i % R);
        const int64_t row = (int64_t)pe[p] * R + r;
        float v = dot(l.gu, row, xp + (int64_t)pb[p] * d_, act_quant_ ? &qx[pb[p]] : nullptr, tmp.data());
        if (!l.bgu.empty()) v += l.bgu[row];
        gu[(size_t)i] = v;
      }
    });
    for (int p = 0; p < P; p++)
      for (int c = 0; c < f_; c++) {
        const int blk = c / 8, off = c % 8;
        const float g = gu[(size_t)p * R + blk * 16 + off], u = gu[(size_t)p * R + blk * 16 + 8 + off];
        h[(size_t)p * f_ + c] = gated(g, u);
      }
    std::vector<QAct> qh(act_quant_ ? P : 0);
    for (int p = 0; p < (int)qh.size(); p++) qh[p].build(h.data() + (size_t)p * f_, f_);
    pool().parallel_for((int64_t)P * d_, [&](int64_t i0, int64_t i1) {
      std::vector<float> tmp(f_);
      for (int64_t i = i0; i < i1; i++) {
        const int p = (int)(i / d_), r = (int)(i % d_);
        const int64_t row = (int64_t)pe[p] * d_ + r;
        float v = dot(l.dn, row, h.data() + (size_t)p * f_, act_quant_ ? &qh[p] : nullptr, tmp.data());
        if (!l.bdn.empty()) v += l.bdn[row];
        y[(size_t)i] = v;
      }
    });
    for (int p = 0; p < P; p++) {   // slots in (token, slot) order
      float* o = op + (int64_t)pb[p] * d_;
      for (int c = 0; c < d_; c++) o[c] += pw[p] * y[(size_t)p * d_ + c];
    }
  }

  int64_t bytes() const {
    int64_t n = 0;
    for (const L& l : layers_) n += (int64_t)l.gu.raw.size() + (int64_t)l.dn.raw.size();
    return n;
  }

 private:
  struct L {
    int e0 = 0, n = 0;
    Mat gu, dn;
    std::vector<float> bgu, bdn;
  };

  static void load(Mat& m, const torch::Tensor& t, int qt, int rows, int cols) {
    if (t.is_cuda() || t.scalar_type() != torch::kUInt8 || !t.is_contiguous())
      throw std::runtime_error("CpuExperts: host uint8 rows");
    const int64_t rb = row_bytes_of(qt, cols);
    if (t.numel() != (int64_t)rows * rb)
      throw std::runtime_error("CpuExperts: expected " + std::to_string(rows) + " rows of " + std::to_string(rb) +
                               " bytes");
    m.qt = qt;
    m.rows = rows;
    m.cols = cols;
    m.row_bytes = rb;
    m.raw.assign(t.data_ptr<uint8_t>(), t.data_ptr<uint8_t>() + t.numel());
  }
  static std::vector<float> floats(const torch::Tensor& t, int64_t n) {
    if (t.is_cuda() || t.scalar_type() != torch::kFloat32 || !t.is_contiguous() || t.numel() != n)
      throw std::runtime_error("CpuExperts: bias of " + std::to_string(n) + " host floats");
    return std::vector<float>(t.data_ptr<float>(), t.data_ptr<float>() + n);
  }
  // one row of m dotted with x: int8 x int8 per 32-block for Q8_0 rows when the activations are
  // quantized, else the row dequantized and dotted in double
  static float dot(const Mat& m, int64_t r, const float* x, const QAct* qa, float* tmp) {
    const uint8_t* row = m.raw.data() + r * m.row_bytes;
    if (qa && m.qt == Q8_0) {
      float acc = 0.f;
      for (int b = 0; b < m.cols / 32; b++) {
        const uint8_t* blk = row + b * 34;
        const int8_t* wq = reinterpret_cast<const int8_t*>(blk + 2);
        const int8_t* xq = qa->q.data() + b * 32;
        int s = 0;
        for (int i = 0; i < 32; i++) s += (int)wq[i] * (int)xq[i];
        acc += h2f(rd16(blk)) * qa->d[b] * (float)s;
      }
      return acc;
    }
    dequant_row(m, (int)r, tmp);
    double acc = 0.0;
    for (int i = 0; i < m.cols; i++) acc += (double)tmp[i] * (double)x[i];
    return (float)acc;
  }
  float gated(float g, float u) const {
    if (gate_ == 4) {   // gpt-oss: alpha 1.702, limit 7
      g = std::min(g, 7.f);
      u = std::min(std::max(u, -7.f), 7.f);
      return (u + 1.f) * g / (1.f + std::exp(-1.702f * g));
    }
    if (gate_ == 3) {   // GELU, tanh form
      const float t = std::tanh(0.7978845608f * (g + 0.044715f * g * g * g));
      return 0.5f * g * (1.f + t) * u;
    }
    return g / (1.f + std::exp(-g)) * u;
  }

  int d_, f_, gate_;
  bool act_quant_;
  std::vector<L> layers_;
};

void register_radix(py::module& m);

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "fak_b200 C++ CPU runtime: GGUF-block decoder forward (oracle + CPU serving path)";
  py::class_<CpuModel>(m, "CpuModel")
      .def(py::init<py::dict, bool>(), py::arg("cfg"), py::arg("act_quant") = true)
      .def("set_matrix", &CpuModel::set_matrix)
      .def("set_vector", &CpuModel::set_vector)
      .def("reset", &CpuModel::reset)
      .def("step", &CpuModel::step, py::call_guard<py::gil_scoped_release>())
      .def("generate", &CpuModel::generate, py::call_guard<py::gil_scoped_release>())
      .def("threads", &CpuModel::threads);
  py::class_<CpuExperts>(m, "CpuExperts")
      .def(py::init<int64_t, int64_t, int64_t, int64_t, bool>(), py::arg("n_layers"), py::arg("d"), py::arg("f"),
           py::arg("gate"), py::arg("act_quant") = true)
      .def("set_layer", &CpuExperts::set_layer, py::arg("layer"), py::arg("e0"), py::arg("n"), py::arg("gate_up"),
           py::arg("qt_gu"), py::arg("down"), py::arg("qt_dn"), py::arg("bias_gu") = py::none(),
           py::arg("bias_dn") = py::none())
      .def("ffn", &CpuExperts::ffn)
      .def("bytes", &CpuExperts::bytes);
  register_radix(m);
}

// oracle.cpp — CPU restatement of the reference crate's tensor lenses.
//
// TEST INFRASTRUCTURE ONLY.  This file is the oracle the CUDA path is checked
// against; it is never linked into libdop.so and no product code path calls
// it.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm may
// load liboracle.so.
//
// It restates, loop for loop and in the same f32 accumulation order, the Rust
// functions of dependent-optics:
//   src/mixtral.rs:126-185  layout / parameter_count
//   src/mixtral.rs:291-380  forward_layer
//   src/mixtral.rs:434-598  backward_layer
//   src/mixtral.rs:238-289,382-432  forward_backward / forward / backward
//   src/mixtral.rs:600-1001 helpers (embed, linear, rmsnorm, rope, gqa,
//                           softmax, topk_renorm, silu, cross_entropy, sgd)
//   src/kernel.rs:173-447   Program forward/backward, gemm, attention
// The crate is Rust-only and cannot be compiled here (no cargo/rustc), so
// parity of this restatement is pinned by the crate's own tests restated in
// tests/test_oracle.py (finite differences, zero gradient of unselected
// experts, SGD descent, tape sizes, parameter counts) and by an independent
// torch-autograd model of the same block in float64.
//
// Build: compiled by oracle/Makefile with -O3 -ffp-contract=off and no
// fast-math, so that, like rustc, no multiply-add is fused and no sum is
// reassociated.  Rust's f32 exp/ln/powf/sin_cos/sqrt call the platform libm;
// this file calls the same libm entry points.  Loop nests are interchanged
// and threaded only where every output keeps the crate's accumulation
// sequence (see `g_literal` below); orc_set_literal(1) runs the crate's
// literal loop order instead, and the two give the same bytes.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <thread>
#include <vector>

#include "../include/dop.h"

typedef std::vector<float> vecf;

namespace {

struct Cfg {
  int64_t vocab, dim, layers, heads, kv_heads, head_dim, inter, experts, top_k;
  float eps, theta;
  int64_t window;
  explicit Cfg(const dop_mixtral_cfg* c)
      : vocab(c->vocab), dim(c->dim), layers(c->layers), heads(c->heads),
        kv_heads(c->kv_heads), head_dim(c->head_dim), inter(c->intermediate),
        experts(c->experts), top_k(c->top_k), eps(c->rms_eps),
        theta(c->rope_theta), window(c->sliding_window) {}
  int64_t q_dim() const { return heads * head_dim; }
  int64_t kv_dim() const { return kv_heads * head_dim; }
  int64_t group() const { return heads / kv_heads; }
};

// LayerLayout relative to the start of the layer slice (src/mixtral.rs:135-171).
struct LL {
  int64_t attn_norm, q, k, v, o, ffn_norm, router;
  std::vector<int64_t> gate, up, down;
  int64_t total;
};

LL layer_layout(const Cfg& c) {
  LL l;
  int64_t at = 0;
  l.attn_norm = at; at += c.dim;
  l.q = at; at += c.dim * c.q_dim();
  l.k = at; at += c.dim * c.kv_dim();
  l.v = at; at += c.dim * c.kv_dim();
  l.o = at; at += c.q_dim() * c.dim;
  l.ffn_norm = at; at += c.dim;
  l.router = at; at += c.dim * c.experts;
  for (int64_t e = 0; e < c.experts; ++e) {
    l.gate.push_back(at); at += c.dim * c.inter;
    l.up.push_back(at); at += c.dim * c.inter;
    l.down.push_back(at); at += c.inter * c.dim;
  }
  l.total = at;
  return l;
}

// Loop order.  The crate's `linear`/`linear_bwd` walk the weight matrix
// column by column (stride dout); restated literally that takes minutes per
// token at the Mixtral-8x7B widths.  By default the loop nests below are
// interchanged and split over OpenMP threads ONLY where every output keeps
// the crate's accumulation sequence: each y[m][o] still starts at 0.0f and
// adds x[m][k] * w[k][o] for k = 0, 1, ... in order, each dw[k][o] adds its
// terms for m = 0, 1, ... in order, and reductions over a contiguous index
// (dx) are still one sequential sum per output.  Without -ffast-math and with
// -ffp-contract=off the results are therefore bit-identical to the literal
// loops, which orc_set_literal(1) selects (tests/test_oracle.py compares the
// two modes byte for byte).
int g_literal = 0;
int g_threads = 0;  // 0: every hardware thread

int oracle_threads() {
  if (g_threads > 0) return g_threads;
  unsigned h = std::thread::hardware_concurrency();
  return h ? (int)h : 1;
}

// f(i) for i in [0, n): in order on this thread when `par` is false (or in
// literal mode), else on up to oracle_threads() threads taking grains of
// consecutive indices.  Callers only split work whose outputs are disjoint.
template <class F>
void par_for(int64_t n, bool par, F&& f) {
  int nt = oracle_threads();
  if (!par || g_literal || nt <= 1 || n <= 1) {
    for (int64_t i = 0; i < n; ++i) f(i);
    return;
  }
  const int64_t grain = std::max<int64_t>(1, n / (8 * (int64_t)nt));
  std::atomic<int64_t> next(0);
  auto work = [&]() {
    for (;;) {
      const int64_t i0 = next.fetch_add(grain);
      if (i0 >= n) return;
      const int64_t i1 = std::min(n, i0 + grain);
      for (int64_t i = i0; i < i1; ++i) f(i);
    }
  };
  const int64_t extra = std::min<int64_t>(nt, (n + grain - 1) / grain) - 1;
  std::vector<std::thread> pool;
  for (int64_t t = 0; t < extra; ++t) pool.emplace_back(work);
  work();
  for (auto& t : pool) t.join();
}

// linear (src/mixtral.rs:616-628), literal loop order
vecf linear_lit(const float* x, const float* w, int64_t n, int64_t din, int64_t dout) {
  vecf y(n * dout, 0.0f);
  for (int64_t m = 0; m < n; ++m)
    for (int64_t o = 0; o < dout; ++o) {
      float acc = 0.0f;
      for (int64_t k = 0; k < din; ++k) acc += x[m * din + k] * w[k * dout + o];
      y[m * dout + o] = acc;
    }
  return y;
}

// linear (src/mixtral.rs:616-628): jobs of (8 rows, 128 columns), k ascending
vecf linear(const float* x, const float* w, int64_t n, int64_t din, int64_t dout) {
  if (g_literal) return linear_lit(x, w, n, din, dout);
  vecf y(n * dout, 0.0f);
  const int64_t MB = 8, OB = 128;
  const int64_t nmb = (n + MB - 1) / MB, nob = (dout + OB - 1) / OB;
  float* yp = y.data();
  par_for(nmb * nob, n * din * dout > (1 << 18), [&](int64_t job) {
    const int64_t m0 = (job / nob) * MB, m1 = std::min(n, m0 + MB);
    const int64_t o0 = (job % nob) * OB, o1 = std::min(dout, o0 + OB);
    for (int64_t k = 0; k < din; ++k) {
      const float* wr = w + k * dout;
      for (int64_t m = m0; m < m1; ++m) {
        const float xk = x[m * din + k];
        float* yr = yp + m * dout;
        for (int64_t o = o0; o < o1; ++o) yr[o] += xk * wr[o];
      }
    }
  });
  return y;
}

// linear_bwd (src/mixtral.rs:630-659), literal loop order
void linear_bwd_lit(const float* x, const float* dy, const float* w, int64_t n, int64_t din,
                    int64_t dout, vecf& dx, vecf& dw) {
  dx.assign(n * din, 0.0f);
  dw.assign(din * dout, 0.0f);
  for (int64_t m = 0; m < n; ++m)
    for (int64_t k = 0; k < din; ++k) {
      float acc = 0.0f;
      for (int64_t o = 0; o < dout; ++o) acc += dy[m * dout + o] * w[k * dout + o];
      dx[m * din + k] = acc;
    }
  for (int64_t k = 0; k < din; ++k)
    for (int64_t o = 0; o < dout; ++o) {
      float acc = 0.0f;
      for (int64_t m = 0; m < n; ++m) acc += x[m * din + k] * dy[m * dout + o];
      dw[k * dout + o] = acc;
    }
}

// linear_bwd (src/mixtral.rs:630-659): dx one sequential sum per output;
// dw row k accumulates the rows m = 0, 1, ... in order
void linear_bwd(const float* x, const float* dy, const float* w, int64_t n, int64_t din,
                int64_t dout, vecf& dx, vecf& dw) {
  if (g_literal) return linear_bwd_lit(x, dy, w, n, din, dout, dx, dw);
  dx.assign(n * din, 0.0f);
  dw.assign(din * dout, 0.0f);
  float* dxp = dx.data();
  float* dwp = dw.data();
  const bool par = n * din * dout > (1 << 18);
  par_for(din * n, par, [&](int64_t job) {
    const int64_t k = job / n, m = job % n;
    const float* wr = w + k * dout;
    const float* dyr = dy + m * dout;
    float acc = 0.0f;
    for (int64_t o = 0; o < dout; ++o) acc += dyr[o] * wr[o];
    dxp[m * din + k] = acc;
  });
  par_for(din, par, [&](int64_t k) {
    float* dr = dwp + k * dout;
    for (int64_t m = 0; m < n; ++m) {
      const float xk = x[m * din + k];
      const float* dyr = dy + m * dout;
      for (int64_t o = 0; o < dout; ++o) dr[o] += xk * dyr[o];
    }
  });
}

// The crate's per-token expert adjoint: linear_bwd on one row (n = 1)
// followed by add_assign of its dw into `grad` (src/mixtral.rs:463-475).
// The dw of one row is the single product 0.0f + x[k] * dy[o]; the default
// mode adds that same value into grad in the same pass.
void linear_bwd_row_acc(const float* x, const float* dy, const float* w, int64_t din,
                        int64_t dout, vecf& dx, float* grad) {
  if (g_literal) {
    vecf dw;
    linear_bwd_lit(x, dy, w, 1, din, dout, dx, dw);
    for (int64_t i = 0; i < din * dout; ++i) grad[i] += dw[i];
    return;
  }
  dx.assign(din, 0.0f);
  float* dxp = dx.data();
  par_for(din, din * dout > (1 << 18), [&](int64_t k) {
    const float* wr = w + k * dout;
    float acc = 0.0f;
    for (int64_t o = 0; o < dout; ++o) acc += dy[o] * wr[o];
    dxp[k] = acc;
    const float xk = x[k];
    float* g = grad + k * dout;
    for (int64_t o = 0; o < dout; ++o) {
      const float p = xk * dy[o];
      g[o] += 0.0f + p;
    }
  });
}

// add_assign (src/mixtral.rs:661-665)
void add_assign(float* dst, const float* src, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] += src[i];
}

// rmsnorm (src/mixtral.rs:667-684): r = sqrt(mean + eps).recip()
void rmsnorm(const float* x, const float* w, int64_t n, int64_t dim, float eps, vecf& y,
             vecf& inv) {
  y.assign(n * dim, 0.0f);
  inv.assign(n, 0.0f);
  for (int64_t t = 0; t < n; ++t) {
    float mean = 0.0f;
    for (int64_t i = 0; i < dim; ++i) {
      float v = x[t * dim + i];
      mean += v * v;
    }
    mean = mean / (float)dim + eps;
    float r = 1.0f / std::sqrt(mean);
    inv[t] = r;
    for (int64_t i = 0; i < dim; ++i) y[t * dim + i] = x[t * dim + i] * r * w[i];
  }
}

// rmsnorm_out (src/mixtral.rs:686-694)
vecf rmsnorm_out(const float* x, const float* inv, const float* w, int64_t n, int64_t dim) {
  vecf y(n * dim, 0.0f);
  for (int64_t t = 0; t < n; ++t)
    for (int64_t i = 0; i < dim; ++i) y[t * dim + i] = x[t * dim + i] * inv[t] * w[i];
  return y;
}

// rmsnorm_bwd (src/mixtral.rs:696-723)
void rmsnorm_bwd(const float* dy, const float* x, const float* inv, const float* w, int64_t n,
                 int64_t dim, vecf& dx, vecf& dw) {
  dx.assign(n * dim, 0.0f);
  dw.assign(dim, 0.0f);
  for (int64_t t = 0; t < n; ++t) {
    float r = inv[t];
    float dot = 0.0f;
    for (int64_t i = 0; i < dim; ++i) {
      float xhat = x[t * dim + i] * r;
      float dxhat = dy[t * dim + i] * w[i];
      dw[i] += dy[t * dim + i] * xhat;
      dot += dxhat * xhat;
    }
    float mean = dot / (float)dim;
    for (int64_t i = 0; i < dim; ++i) {
      float xhat = x[t * dim + i] * r;
      float dxhat = dy[t * dim + i] * w[i];
      dx[t * dim + i] = r * (dxhat - xhat * mean);
    }
  }
}

// rope_angles (src/mixtral.rs:725-739)
void rope_angles(const Cfg& c, int64_t pos, vecf& cs, vecf& sn) {
  int64_t half = c.head_dim / 2;
  cs.assign(c.head_dim, 0.0f);
  sn.assign(c.head_dim, 0.0f);
  for (int64_t i = 0; i < half; ++i) {
    float freq = std::pow(c.theta, -(2.0f * (float)i) / (float)c.head_dim);
    float ang = (float)pos * freq;
    float s = std::sin(ang), co = std::cos(ang);
    cs[i] = co; cs[half + i] = co;
    sn[i] = s; sn[half + i] = s;
  }
}

// rope_qkv / rope_qkv_transpose (src/mixtral.rs:741-797); sign = +1 / -1
vecf rope(const Cfg& c, const float* src, int64_t n_elems, int64_t batch, int64_t seq,
          int64_t n_heads, float sign) {
  int64_t hd = c.head_dim, half = hd / 2;
  vecf y(n_elems, 0.0f);
  vecf cs, sn;
  for (int64_t b = 0; b < batch; ++b)
    for (int64_t t = 0; t < seq; ++t) {
      rope_angles(c, t, cs, sn);
      for (int64_t h = 0; h < n_heads; ++h) {
        int64_t base = ((b * seq + t) * n_heads + h) * hd;
        for (int64_t i = 0; i < half; ++i) {
          float q1 = src[base + i], q2 = src[base + half + i];
          float s = sign * sn[i];
          y[base + i] = q1 * cs[i] - q2 * s;
          y[base + half + i] = q2 * cs[half + i] + q1 * s;
        }
      }
    }
  return y;
}

// visible (src/mixtral.rs:799-801)
inline bool visible(const Cfg& c, int64_t q, int64_t k) { return k <= q && q - k < c.window; }

// gqa_forward (src/mixtral.rs:803-859)
void gqa_forward(const Cfg& c, const float* q, const float* k, const float* v, int64_t batch,
                 int64_t seq, vecf& probs, vecf& mix) {
  int64_t hd = c.head_dim;
  float scale = 1.0f / std::sqrt((float)hd);
  int64_t group = c.group();
  probs.assign(batch * c.heads * seq * seq, 0.0f);
  mix.assign(batch * seq * c.q_dim(), 0.0f);
  // (b, h) rows are independent: split over threads, each row computed as
  // the crate computes it
  par_for(batch * c.heads, true, [&](int64_t bh) {
    const int64_t b = bh / c.heads, h = bh % c.heads;
    vecf row(seq);
    {
      int64_t kv = h / group;
      for (int64_t i = 0; i < seq; ++i) {
        std::fill(row.begin(), row.end(), -INFINITY);
        float max_s = -INFINITY;
        for (int64_t j = 0; j < seq; ++j) {
          if (!visible(c, i, j)) continue;
          float dot = 0.0f;
          for (int64_t d = 0; d < hd; ++d)
            dot += q[((b * seq + i) * c.heads + h) * hd + d] *
                   k[((b * seq + j) * c.kv_heads + kv) * hd + d];
          row[j] = dot * scale;
          max_s = std::max(max_s, row[j]);  // f32::max: NaN-ignoring, same for finite
        }
        float sum = 0.0f;
        for (int64_t j = 0; j < seq; ++j) {
          if (std::isfinite(row[j])) {
            row[j] = std::exp(row[j] - max_s);
            sum += row[j];
          } else {
            row[j] = 0.0f;
          }
        }
        for (int64_t j = 0; j < seq; ++j) {
          row[j] /= sum;
          probs[((b * c.heads + h) * seq + i) * seq + j] = row[j];
        }
        for (int64_t d = 0; d < hd; ++d) {
          float acc = 0.0f;
          for (int64_t j = 0; j < seq; ++j)
            acc += row[j] * v[((b * seq + j) * c.kv_heads + kv) * hd + d];
          mix[((b * seq + i) * c.heads + h) * hd + d] = acc;
        }
      }
    }
  });
}

// gqa_backward (src/mixtral.rs:861-922)
void gqa_backward(const Cfg& c, const float* q, const float* k, const float* v,
                  const float* probs, const float* dmix, int64_t batch, int64_t seq,
                  int64_t q_len, int64_t kv_len, vecf& dq, vecf& dk, vecf& dv) {
  int64_t hd = c.head_dim;
  float scale = 1.0f / std::sqrt((float)hd);
  int64_t group = c.group();
  dq.assign(q_len, 0.0f);
  dk.assign(kv_len, 0.0f);
  dv.assign(kv_len, 0.0f);
  // dk/dv of KV head kvh receive only the heads of its group: (b, kvh) pairs
  // are split over threads and each walks its heads in the crate's order
  par_for(batch * c.kv_heads, true, [&](int64_t bg) {
    const int64_t b = bg / c.kv_heads;
    vecf da(seq);
    for (int64_t h = (bg % c.kv_heads) * group; h < (bg % c.kv_heads + 1) * group; ++h) {
      int64_t kvh = h / group;
      for (int64_t i = 0; i < seq; ++i) {
        std::fill(da.begin(), da.end(), 0.0f);
        const float* prow = probs + ((b * c.heads + h) * seq + i) * seq;
        for (int64_t j = 0; j < seq; ++j) {
          if (prow[j] == 0.0f && !visible(c, i, j)) continue;
          float dot = 0.0f;
          for (int64_t d = 0; d < hd; ++d)
            dot += dmix[((b * seq + i) * c.heads + h) * hd + d] *
                   v[((b * seq + j) * c.kv_heads + kvh) * hd + d];
          da[j] = dot;
          float p = prow[j];
          for (int64_t d = 0; d < hd; ++d)
            dv[((b * seq + j) * c.kv_heads + kvh) * hd + d] +=
                p * dmix[((b * seq + i) * c.heads + h) * hd + d];
        }
        float dot_pa = 0.0f;
        for (int64_t j = 0; j < seq; ++j) dot_pa += prow[j] * da[j];
        for (int64_t j = 0; j < seq; ++j) {
          if (!visible(c, i, j)) continue;
          float p = prow[j];
          float ds = p * (da[j] - dot_pa) * scale;
          for (int64_t d = 0; d < hd; ++d) {
            dq[((b * seq + i) * c.heads + h) * hd + d] +=
                ds * k[((b * seq + j) * c.kv_heads + kvh) * hd + d];
            dk[((b * seq + j) * c.kv_heads + kvh) * hd + d] +=
                ds * q[((b * seq + i) * c.heads + h) * hd + d];
          }
        }
      }
    }
  });
}

// softmax (src/mixtral.rs:924-929)
vecf softmax(const float* z, int64_t n) {
  float m = -INFINITY;
  for (int64_t i = 0; i < n; ++i) m = std::max(m, z[i]);
  vecf e(n);
  for (int64_t i = 0; i < n; ++i) e[i] = std::exp(z[i] - m);
  float s = 0.0f;
  for (int64_t i = 0; i < n; ++i) s += e[i];
  for (int64_t i = 0; i < n; ++i) e[i] = e[i] / s;
  return e;
}

// topk_renorm (src/mixtral.rs:931-939): prob descending, then index ascending
void topk_renorm(const vecf& probs, int64_t k, std::vector<int64_t>& idx, vecf& p, vecf& w) {
  int64_t n = (int64_t)probs.size();
  idx.resize(n);
  for (int64_t i = 0; i < n; ++i) idx[i] = i;
  std::stable_sort(idx.begin(), idx.end(), [&](int64_t a, int64_t b) {
    if (probs[b] != probs[a]) return probs[a] > probs[b];
    return a < b;
  });
  idx.resize(k);
  p.resize(k);
  for (int64_t i = 0; i < k; ++i) p[i] = probs[idx[i]];
  float s = 0.0f;
  for (int64_t i = 0; i < k; ++i) s += p[i];
  w.resize(k);
  for (int64_t i = 0; i < k; ++i) w[i] = p[i] / s;
}

// sigmoid / silu / silu_mul / silu_mul_bwd (src/mixtral.rs:941-964)
inline float sigmoid(float z) { return 1.0f / (1.0f + std::exp(-z)); }
inline float silu(float z) { return z * sigmoid(z); }

}  // namespace

// LayerTape (src/mixtral.rs:212-228)
struct orc_tape {
  Cfg cfg;
  int64_t batch, seq;
  vecf attn_in, attn_inv, q_pre, k_pre, v, probs, mix, ffn_in, ffn_inv, router_probs;
  std::vector<int64_t> top_i;
  vecf top_p, top_w, gate, up;
  explicit orc_tape(const dop_mixtral_cfg* c) : cfg(c) {}
};

namespace {

// forward_layer (src/mixtral.rs:291-380).  `lp` is the layer slice; `bias`
// (may be null) is added to the router logits (skewed-routing workload only).
vecf forward_layer(const Cfg& c, const float* lp, const float* x, int64_t batch, int64_t seq,
                   orc_tape& lt, const float* bias, const int64_t* forced_top_i = nullptr) {
  LL L = layer_layout(c);
  int64_t n = batch * seq;
  vecf xn, attn_inv;
  rmsnorm(x, lp + L.attn_norm, n, c.dim, c.eps, xn, attn_inv);
  vecf q_pre = linear(xn.data(), lp + L.q, n, c.dim, c.q_dim());
  vecf k_pre = linear(xn.data(), lp + L.k, n, c.dim, c.kv_dim());
  vecf v = linear(xn.data(), lp + L.v, n, c.dim, c.kv_dim());
  vecf q = rope(c, q_pre.data(), (int64_t)q_pre.size(), batch, seq, c.heads, 1.0f);
  vecf k = rope(c, k_pre.data(), (int64_t)k_pre.size(), batch, seq, c.kv_heads, 1.0f);
  vecf probs, mix;
  gqa_forward(c, q.data(), k.data(), v.data(), batch, seq, probs, mix);
  vecf attn = linear(mix.data(), lp + L.o, n, c.q_dim(), c.dim);
  vecf mid(x, x + n * c.dim);
  add_assign(mid.data(), attn.data(), n * c.dim);

  vecf xn2, ffn_inv;
  rmsnorm(mid.data(), lp + L.ffn_norm, n, c.dim, c.eps, xn2, ffn_inv);
  vecf router_logits = linear(xn2.data(), lp + L.router, n, c.dim, c.experts);
  if (bias)
    for (int64_t t = 0; t < n; ++t)
      for (int64_t e = 0; e < c.experts; ++e) router_logits[t * c.experts + e] += bias[e];
  vecf router_probs(n * c.experts, 0.0f);
  std::vector<int64_t> top_i(n * c.top_k, 0);
  vecf top_p(n * c.top_k, 0.0f), top_w(n * c.top_k, 0.0f);
  std::vector<int64_t> idx;
  vecf p, w;
  for (int64_t t = 0; t < n; ++t) {
    vecf row = softmax(router_logits.data() + t * c.experts, c.experts);
    std::copy(row.begin(), row.end(), router_probs.begin() + t * c.experts);
    topk_renorm(row, c.top_k, idx, p, w);
    if (forced_top_i) {
      // Test hook: take the selection from the caller (the device lens's
      // decision at a near-tie) and renormalise exactly as topk_renorm does.
      float sf = 0.0f;
      for (int64_t k2 = 0; k2 < c.top_k; ++k2) {
        idx[k2] = forced_top_i[t * c.top_k + k2];
        p[k2] = row[idx[k2]];
      }
      for (int64_t k2 = 0; k2 < c.top_k; ++k2) sf += p[k2];
      for (int64_t k2 = 0; k2 < c.top_k; ++k2) w[k2] = p[k2] / sf;
    }
    for (int64_t k2 = 0; k2 < c.top_k; ++k2) {
      top_i[t * c.top_k + k2] = idx[k2];
      top_p[t * c.top_k + k2] = p[k2];
      top_w[t * c.top_k + k2] = w[k2];
    }
  }
  vecf gate(n * c.top_k * c.inter, 0.0f), up(n * c.top_k * c.inter, 0.0f);
  vecf mixed(n * c.dim, 0.0f);
  vecf hid(c.inter);
  for (int64_t t = 0; t < n; ++t)
    for (int64_t k2 = 0; k2 < c.top_k; ++k2) {
      int64_t e = top_i[t * c.top_k + k2];
      const float* xr = xn2.data() + t * c.dim;
      vecf g = linear(xr, lp + L.gate[e], 1, c.dim, c.inter);
      vecf u = linear(xr, lp + L.up[e], 1, c.dim, c.inter);
      for (int64_t i = 0; i < c.inter; ++i) hid[i] = silu(g[i]) * u[i];
      vecf out = linear(hid.data(), lp + L.down[e], 1, c.inter, c.dim);
      float wt = top_w[t * c.top_k + k2];
      for (int64_t d = 0; d < c.dim; ++d) mixed[t * c.dim + d] += wt * out[d];
      int64_t base = (t * c.top_k + k2) * c.inter;
      std::copy(g.begin(), g.end(), gate.begin() + base);
      std::copy(u.begin(), u.end(), up.begin() + base);
    }
  vecf y = mid;
  add_assign(y.data(), mixed.data(), n * c.dim);

  lt.batch = batch;
  lt.seq = seq;
  lt.attn_in.assign(x, x + n * c.dim);
  lt.attn_inv = std::move(attn_inv);
  lt.q_pre = std::move(q_pre);
  lt.k_pre = std::move(k_pre);
  lt.v = std::move(v);
  lt.probs = std::move(probs);
  lt.mix = std::move(mix);
  lt.ffn_in = std::move(mid);
  lt.ffn_inv = std::move(ffn_inv);
  lt.router_probs = std::move(router_probs);
  lt.top_i = std::move(top_i);
  lt.top_p = std::move(top_p);
  lt.top_w = std::move(top_w);
  lt.gate = std::move(gate);
  lt.up = std::move(up);
  return y;
}

// backward_layer (src/mixtral.rs:434-598); `grad` is the layer slice of dP.
vecf backward_layer(const Cfg& c, const float* lp, const orc_tape& lt, const float* dy,
                    float* grad) {
  LL L = layer_layout(c);
  int64_t batch = lt.batch, seq = lt.seq, n = batch * seq;
  const float* d_mixed = dy;
  vecf xn2 = rmsnorm_out(lt.ffn_in.data(), lt.ffn_inv.data(), lp + L.ffn_norm, n, c.dim);
  vecf d_xn2(n * c.dim, 0.0f);
  vecf hid(c.inter), d_out(c.dim), d_gate(c.inter), d_up(c.inter);
  vecf d_hid, dx_g, dx_u, dx_r;
  for (int64_t t = 0; t < n; ++t) {
    vecf dvalues(c.top_k, 0.0f);
    float weight_dot = 0.0f;
    float s = 0.0f;
    for (int64_t k2 = 0; k2 < c.top_k; ++k2) s += lt.top_p[t * c.top_k + k2];
    for (int64_t k2 = 0; k2 < c.top_k; ++k2) {
      int64_t e = lt.top_i[t * c.top_k + k2];
      int64_t base = (t * c.top_k + k2) * c.inter;
      const float* g = lt.gate.data() + base;
      const float* u = lt.up.data() + base;
      for (int64_t i = 0; i < c.inter; ++i) hid[i] = silu(g[i]) * u[i];
      vecf out = linear(hid.data(), lp + L.down[e], 1, c.inter, c.dim);
      float dw = 0.0f;
      for (int64_t d = 0; d < c.dim; ++d) dw += d_mixed[t * c.dim + d] * out[d];
      weight_dot += dw * lt.top_w[t * c.top_k + k2];
      dvalues[k2] = dw;
      float w = lt.top_w[t * c.top_k + k2];
      for (int64_t d = 0; d < c.dim; ++d) d_out[d] = w * d_mixed[t * c.dim + d];
      linear_bwd_row_acc(hid.data(), d_out.data(), lp + L.down[e], c.inter, c.dim, d_hid,
                         grad + L.down[e]);
      for (int64_t i = 0; i < c.inter; ++i) {
        float z = g[i];
        float sg = sigmoid(z);
        float dsilu = sg * (1.0f + z * (1.0f - sg));
        d_gate[i] = d_hid[i] * u[i] * dsilu;
        d_up[i] = d_hid[i] * silu(z);
      }
      const float* xrow = xn2.data() + t * c.dim;
      linear_bwd_row_acc(xrow, d_gate.data(), lp + L.gate[e], c.dim, c.inter, dx_g,
                         grad + L.gate[e]);
      linear_bwd_row_acc(xrow, d_up.data(), lp + L.up[e], c.dim, c.inter, dx_u,
                         grad + L.up[e]);
      for (int64_t d = 0; d < c.dim; ++d) d_xn2[t * c.dim + d] += dx_g[d] + dx_u[d];
    }
    for (int64_t k2 = 0; k2 < c.top_k; ++k2) dvalues[k2] = dvalues[k2] / s - weight_dot / s;
    vecf dp(c.experts, 0.0f);
    for (int64_t k2 = 0; k2 < c.top_k; ++k2) dp[lt.top_i[t * c.top_k + k2]] = dvalues[k2];
    const float* p = lt.router_probs.data() + t * c.experts;
    float dot = 0.0f;
    for (int64_t e = 0; e < c.experts; ++e) dot += p[e] * dp[e];
    vecf dz(c.experts, 0.0f);
    for (int64_t e = 0; e < c.experts; ++e) dz[e] = p[e] * (dp[e] - dot);
    const float* xrow = xn2.data() + t * c.dim;
    linear_bwd_row_acc(xrow, dz.data(), lp + L.router, c.dim, c.experts, dx_r,
                       grad + L.router);
    for (int64_t d = 0; d < c.dim; ++d) d_xn2[t * c.dim + d] += dx_r[d];
  }
  vecf d_mid, d_ffn_w;
  rmsnorm_bwd(d_xn2.data(), lt.ffn_in.data(), lt.ffn_inv.data(), lp + L.ffn_norm, n, c.dim,
              d_mid, d_ffn_w);
  add_assign(grad + L.ffn_norm, d_ffn_w.data(), c.dim);
  add_assign(d_mid.data(), dy, n * c.dim);

  vecf d_mix, d_o;
  linear_bwd(lt.mix.data(), d_mid.data(), lp + L.o, n, c.q_dim(), c.dim, d_mix, d_o);
  add_assign(grad + L.o, d_o.data(), c.q_dim() * c.dim);
  vecf q = rope(c, lt.q_pre.data(), (int64_t)lt.q_pre.size(), batch, seq, c.heads, 1.0f);
  vecf k = rope(c, lt.k_pre.data(), (int64_t)lt.k_pre.size(), batch, seq, c.kv_heads, 1.0f);
  vecf dq, dk, dv;
  gqa_backward(c, q.data(), k.data(), lt.v.data(), lt.probs.data(), d_mix.data(), batch, seq,
               (int64_t)q.size(), (int64_t)k.size(), dq, dk, dv);
  dq = rope(c, dq.data(), (int64_t)dq.size(), batch, seq, c.heads, -1.0f);
  dk = rope(c, dk.data(), (int64_t)dk.size(), batch, seq, c.kv_heads, -1.0f);
  vecf xn = rmsnorm_out(lt.attn_in.data(), lt.attn_inv.data(), lp + L.attn_norm, n, c.dim);
  vecf dx_q, dw_q, dx_k, dw_k, dx_v, dw_v;
  linear_bwd(xn.data(), dq.data(), lp + L.q, n, c.dim, c.q_dim(), dx_q, dw_q);
  linear_bwd(xn.data(), dk.data(), lp + L.k, n, c.dim, c.kv_dim(), dx_k, dw_k);
  linear_bwd(xn.data(), dv.data(), lp + L.v, n, c.dim, c.kv_dim(), dx_v, dw_v);
  add_assign(grad + L.q, dw_q.data(), c.dim * c.q_dim());
  add_assign(grad + L.k, dw_k.data(), c.dim * c.kv_dim());
  add_assign(grad + L.v, dw_v.data(), c.dim * c.kv_dim());
  vecf d_xn = dx_q;
  add_assign(d_xn.data(), dx_k.data(), n * c.dim);
  add_assign(d_xn.data(), dx_v.data(), n * c.dim);
  vecf dx, d_attn_w;
  rmsnorm_bwd(d_xn.data(), lt.attn_in.data(), lt.attn_inv.data(), lp + L.attn_norm, n, c.dim,
              dx, d_attn_w);
  add_assign(grad + L.attn_norm, d_attn_w.data(), c.dim);
  add_assign(dx.data(), d_mid.data(), n * c.dim);
  return dx;
}

// cross_entropy (src/mixtral.rs:966-991)
float cross_entropy(const float* logits, const int64_t* targets, int64_t n, int64_t vocab,
                    vecf& d) {
  d.assign(n * vocab, 0.0f);
  float loss = 0.0f;
  for (int64_t t = 0; t < n; ++t) {
    const float* row = logits + t * vocab;
    float m = -INFINITY;
    for (int64_t v = 0; v < vocab; ++v) m = std::max(m, row[v]);
    float sum = 0.0f;
    for (int64_t v = 0; v < vocab; ++v) sum += std::exp(row[v] - m);
    float lse = m + std::log(sum);
    loss += lse - row[targets[t]];
    for (int64_t v = 0; v < vocab; ++v)
      d[t * vocab + v] = (std::exp(row[v] - m) / sum) / (float)n;
    d[t * vocab + targets[t]] -= 1.0f / (float)n;
  }
  return loss / (float)n;
}

}  // namespace

// ------------------------------------------------------------------ C ABI
extern "C" {

int64_t orc_layer_params(const dop_mixtral_cfg* c) { return layer_layout(Cfg(c)).total; }

// 1: the crate's literal loop order, single-threaded; 0 (default): the
// interchanged, threaded loop nests (same bytes).
void orc_set_literal(int on) { g_literal = on ? 1 : 0; }

// Host threads the oracle may use (0 = every hardware thread); returns the
// number in effect.
int orc_set_threads(int n) {
  if (n >= 0) g_threads = n;
  return oracle_threads();
}

// offsets out[0..7) = attn_norm,q,k,v,o,ffn_norm,router; then gate[E],up[E],down[E]
void orc_layer_offsets(const dop_mixtral_cfg* c, int64_t* out) {
  Cfg cfg(c);
  LL L = layer_layout(cfg);
  int64_t v[7] = {L.attn_norm, L.q, L.k, L.v, L.o, L.ffn_norm, L.router};
  for (int i = 0; i < 7; ++i) out[i] = v[i];
  for (int64_t e = 0; e < cfg.experts; ++e) {
    out[7 + e] = L.gate[e];
    out[7 + cfg.experts + e] = L.up[e];
    out[7 + 2 * cfg.experts + e] = L.down[e];
  }
}

// parameter_count (src/mixtral.rs:183-185): embed + layers + final_norm + lm_head
int64_t orc_parameter_count(const dop_mixtral_cfg* c) {
  Cfg cfg(c);
  return cfg.vocab * cfg.dim + cfg.layers * layer_layout(cfg).total + cfg.dim +
         cfg.dim * cfg.vocab;
}

// `forced_top_i` (may be null) overrides the top-k selection per token; it is
// used only to align the oracle with the device lens where a bf16 rounding of
// the attention half flipped a near-tie.
orc_tape* orc_block_forward(const dop_mixtral_cfg* c, const float* lp, const float* x,
                            int64_t batch, int64_t seq, const float* router_bias,
                            const int64_t* forced_top_i, float* y) {
  orc_tape* lt = new orc_tape(c);
  vecf out = forward_layer(lt->cfg, lp, x, batch, seq, *lt, router_bias, forced_top_i);
  std::memcpy(y, out.data(), out.size() * sizeof(float));
  return lt;
}

void orc_block_backward(const dop_mixtral_cfg* c, const float* lp, const orc_tape* lt,
                        const float* dy, float* dx, float* dlp) {
  Cfg cfg(c);
  vecf out = backward_layer(cfg, lp, *lt, dy, dlp);
  std::memcpy(dx, out.data(), out.size() * sizeof(float));
}

void orc_tape_routing(const orc_tape* lt, int64_t* top_i, float* top_p, float* top_w,
                      float* router_probs) {
  if (top_i) std::copy(lt->top_i.begin(), lt->top_i.end(), top_i);
  if (top_p) std::copy(lt->top_p.begin(), lt->top_p.end(), top_p);
  if (top_w) std::copy(lt->top_w.begin(), lt->top_w.end(), top_w);
  if (router_probs) std::copy(lt->router_probs.begin(), lt->router_probs.end(), router_probs);
}

void orc_tape_free(orc_tape* lt) { delete lt; }

// The router stage of forward_layer on a given feed-forward input `mid`
// [n, D] (src/mixtral.rs:311-327): xn2 = rmsnorm(mid), logits = xn2 Wr
// (+ bias, the skewed-routing workload), softmax, topk_renorm.  Outputs
// top_i/top_p/top_w [n, k] and router_probs [n, E] (any may be null).
void orc_router_stage(const dop_mixtral_cfg* c, const float* lp, const float* mid, int64_t n,
                      const float* bias, int64_t* top_i, float* top_p, float* top_w,
                      float* router_probs) {
  Cfg cfg(c);
  LL L = layer_layout(cfg);
  vecf xn2, inv;
  rmsnorm(mid, lp + L.ffn_norm, n, cfg.dim, cfg.eps, xn2, inv);
  vecf logits = linear(xn2.data(), lp + L.router, n, cfg.dim, cfg.experts);
  if (bias)
    for (int64_t t = 0; t < n; ++t)
      for (int64_t e = 0; e < cfg.experts; ++e) logits[t * cfg.experts + e] += bias[e];
  std::vector<int64_t> idx;
  vecf pk, wk;
  for (int64_t t = 0; t < n; ++t) {
    vecf row = softmax(logits.data() + t * cfg.experts, cfg.experts);
    if (router_probs) std::copy(row.begin(), row.end(), router_probs + t * cfg.experts);
    topk_renorm(row, cfg.top_k, idx, pk, wk);
    for (int64_t k2 = 0; k2 < cfg.top_k; ++k2) {
      if (top_i) top_i[t * cfg.top_k + k2] = idx[k2];
      if (top_p) top_p[t * cfg.top_k + k2] = pk[k2];
      if (top_w) top_w[t * cfg.top_k + k2] = wk[k2];
    }
  }
}

// forward_backward (src/mixtral.rs:245-261) with forward (:263-289) and backward (:382-432).
float orc_mixtral_forward_backward(const dop_mixtral_cfg* c, const float* P,
                                   const int64_t* tokens, const int64_t* targets,
                                   int64_t batch, int64_t seq, float* grad, float* logits) {
  Cfg cfg(c);
  LL L = layer_layout(cfg);
  int64_t n = batch * seq, D = cfg.dim;
  int64_t embed = 0, layer0 = cfg.vocab * D;
  int64_t final_norm = layer0 + cfg.layers * L.total, lm_head = final_norm + D;
  int64_t total = lm_head + D * cfg.vocab;
  // embed (src/mixtral.rs:600-606)
  vecf x(n * D, 0.0f);
  for (int64_t t = 0; t < n; ++t)
    std::copy(P + embed + tokens[t] * D, P + embed + (tokens[t] + 1) * D, x.begin() + t * D);
  std::vector<orc_tape*> tapes;
  for (int64_t l = 0; l < cfg.layers; ++l) {
    orc_tape* lt = new orc_tape(c);
    x = forward_layer(cfg, P + layer0 + l * L.total, x.data(), batch, seq, *lt, nullptr);
    tapes.push_back(lt);
  }
  vecf final_h, final_inv;
  rmsnorm(x.data(), P + final_norm, n, D, cfg.eps, final_h, final_inv);
  vecf lg = linear(final_h.data(), P + lm_head, n, D, cfg.vocab);
  vecf dlogits;
  float loss = cross_entropy(lg.data(), targets, n, cfg.vocab, dlogits);
  std::fill(grad, grad + total, 0.0f);
  vecf hn = rmsnorm_out(x.data(), final_inv.data(), P + final_norm, n, D);
  vecf dx, dhead;
  linear_bwd(hn.data(), dlogits.data(), P + lm_head, n, D, cfg.vocab, dx, dhead);
  add_assign(grad + lm_head, dhead.data(), D * cfg.vocab);
  vecf dxn, dweight;
  rmsnorm_bwd(dx.data(), x.data(), final_inv.data(), P + final_norm, n, D, dxn, dweight);
  dx = dxn;
  add_assign(grad + final_norm, dweight.data(), D);
  for (int64_t l = cfg.layers - 1; l >= 0; --l)
    dx = backward_layer(cfg, P + layer0 + l * L.total, *tapes[l], dx.data(),
                        grad + layer0 + l * L.total);
  // embed_bwd (src/mixtral.rs:608-614)
  for (int64_t t = 0; t < n; ++t)
    for (int64_t d = 0; d < D; ++d) grad[embed + tokens[t] * D + d] += dx[t * D + d];
  for (auto* lt : tapes) delete lt;
  if (logits) std::copy(lg.begin(), lg.end(), logits);
  return loss;
}

// sgd_step (src/mixtral.rs:994-1001); returns the gradient norm
float orc_sgd_step(float* params, const float* grad, int64_t n, float lr) {
  float norm = 0.0f;
  for (int64_t i = 0; i < n; ++i) {
    norm += grad[i] * grad[i];
    params[i] -= lr * grad[i];
  }
  return std::sqrt(norm);
}

// ---------------------------------------------------- kernel.rs programs
// Program forward_backward (src/kernel.rs:181-240) generalised to a given
// upstream cotangent dy0 (NULL = the crate's sum loss, dy = 1), which the
// private `backward(prog, params, tape, mask, dy0)` (src/kernel.rs:293) admits.
void orc_program_forward_backward(const dop_stage* stages, int64_t n_stages, int64_t input_len,
                                  int64_t param_len, int64_t tape_f32, int64_t tape_u8,
                                  const float* x, const float* params, const float* dy0,
                                  float* y_out, int64_t* y_len, float* dx_out, float* dp_out) {
  (void)param_len;
  vecf tape(tape_f32, 0.0f);
  std::vector<uint8_t> mask(tape_u8, 0);
  vecf cur(x, x + input_len);
  for (int64_t si = 0; si < n_stages; ++si) {
    const dop_stage& st = stages[si];
    if (st.kind == DOP_STAGE_GEMM) {
      std::copy(cur.begin(), cur.end(), tape.begin() + st.save_at);
      const float* w = params + st.param_at;
      const float* bias = params + st.param_at + st.din * st.dout;
      // gemm (src/kernel.rs:242-254): acc starts at the bias
      vecf yv(st.batch * st.dout, 0.0f);
      for (int64_t m = 0; m < st.batch; ++m)
        for (int64_t nn = 0; nn < st.dout; ++nn) {
          float acc = bias[nn];
          for (int64_t k = 0; k < st.din; ++k) acc += cur[m * st.din + k] * w[k * st.dout + nn];
          yv[m * st.dout + nn] = acc;
        }
      if (st.relu)
        for (int64_t i = 0; i < (int64_t)yv.size(); ++i) {
          bool on = yv[i] > 0.0f;
          mask[st.mask_at + i] = on ? 1 : 0;
          if (!on) yv[i] = 0.0f;
        }
      cur = yv;
    } else if (st.kind == DOP_STAGE_ATTENTION) {
      std::copy(cur.begin(), cur.end(), tape.begin() + st.x_at);
      // attention_forward (src/kernel.rs:256-291)
      int64_t B = st.batch, T = st.tokens, D = st.dim;
      float scale = 1.0f / std::sqrt((float)D);
      vecf yv(B * T * D, 0.0f), row(T);
      for (int64_t b = 0; b < B; ++b)
        for (int64_t i = 0; i < T; ++i) {
          float max_s = -INFINITY;
          for (int64_t j = 0; j < T; ++j) {
            float dot = 0.0f;
            for (int64_t d = 0; d < D; ++d) dot += cur[(b * T + i) * D + d] * cur[(b * T + j) * D + d];
            row[j] = dot * scale;
            max_s = std::max(max_s, row[j]);
          }
          float sum = 0.0f;
          for (int64_t j = 0; j < T; ++j) {
            row[j] = std::exp(row[j] - max_s);
            sum += row[j];
          }
          for (int64_t j = 0; j < T; ++j) {
            row[j] /= sum;
            tape[st.probs_at + (b * T + i) * T + j] = row[j];
          }
          for (int64_t d = 0; d < D; ++d) {
            float acc = 0.0f;
            for (int64_t j = 0; j < T; ++j) acc += row[j] * cur[(b * T + j) * D + d];
            yv[(b * T + i) * D + d] = acc;
          }
        }
      cur = yv;
    } else {
      for (int64_t i = 0; i < st.len; ++i) cur[i] += tape[st.from + i];
    }
  }
  std::copy(cur.begin(), cur.end(), y_out);
  *y_len = (int64_t)cur.size();

  // backward (src/kernel.rs:293-374)
  vecf dy = dy0 ? vecf(dy0, dy0 + cur.size()) : vecf(cur.size(), 1.0f);
  std::fill(dp_out, dp_out + param_len, 0.0f);
  std::vector<std::pair<int64_t, vecf>> side;
  auto add_side = [&](int64_t at, vecf& dx) {  // add_side (src/kernel.rs:376-388)
    size_t i = 0;
    while (i < side.size()) {
      if (side[i].first == at) {
        for (size_t j = 0; j < dx.size() && j < side[i].second.size(); ++j) dx[j] += side[i].second[j];
        side.erase(side.begin() + i);
      } else {
        ++i;
      }
    }
  };
  for (int64_t si = n_stages - 1; si >= 0; --si) {
    const dop_stage& st = stages[si];
    if (st.kind == DOP_STAGE_ADD) {
      side.emplace_back(st.from, vecf(dy.begin(), dy.begin() + st.len));
    } else if (st.kind == DOP_STAGE_GEMM) {
      if (st.relu)
        for (int64_t i = 0; i < st.batch * st.dout; ++i)
          if (mask[st.mask_at + i] == 0) dy[i] = 0.0f;
      const float* xs = tape.data() + st.save_at;
      const float* w = params + st.param_at;
      vecf dx(st.batch * st.din, 0.0f);
      for (int64_t m = 0; m < st.batch; ++m)
        for (int64_t k = 0; k < st.din; ++k) {
          float acc = 0.0f;
          for (int64_t nn = 0; nn < st.dout; ++nn) acc += dy[m * st.dout + nn] * w[k * st.dout + nn];
          dx[m * st.din + k] = acc;
        }
      for (int64_t k = 0; k < st.din; ++k)
        for (int64_t nn = 0; nn < st.dout; ++nn) {
          float acc = 0.0f;
          for (int64_t m = 0; m < st.batch; ++m) acc += xs[m * st.din + k] * dy[m * st.dout + nn];
          dp_out[st.param_at + k * st.dout + nn] = acc;
        }
      int64_t b_at = st.param_at + st.din * st.dout;
      for (int64_t nn = 0; nn < st.dout; ++nn) {
        float acc = 0.0f;
        for (int64_t m = 0; m < st.batch; ++m) acc += dy[m * st.dout + nn];
        dp_out[b_at + nn] = acc;
      }
      add_side(st.save_at, dx);
      dy = dx;
    } else {
      // attention_backward (src/kernel.rs:390-447)
      int64_t B = st.batch, T = st.tokens, D = st.dim;
      float scale = 1.0f / std::sqrt((float)D);
      const float* xs = tape.data() + st.x_at;
      const float* probs = tape.data() + st.probs_at;
      vecf d_v(B * T * D, 0.0f), d_a(B * T * T, 0.0f);
      for (int64_t b = 0; b < B; ++b)
        for (int64_t i = 0; i < T; ++i)
          for (int64_t j = 0; j < T; ++j) {
            float p = probs[(b * T + i) * T + j];
            float dot = 0.0f;
            for (int64_t d = 0; d < D; ++d) {
              float yy = dy[(b * T + i) * D + d];
              d_v[(b * T + j) * D + d] += p * yy;
              dot += yy * xs[(b * T + j) * D + d];
            }
            d_a[(b * T + i) * T + j] = dot;
          }
      vecf d_s(d_a.size(), 0.0f);
      for (int64_t b = 0; b < B; ++b)
        for (int64_t i = 0; i < T; ++i) {
          float dot = 0.0f;
          for (int64_t j = 0; j < T; ++j) dot += probs[(b * T + i) * T + j] * d_a[(b * T + i) * T + j];
          for (int64_t j = 0; j < T; ++j)
            d_s[(b * T + i) * T + j] = probs[(b * T + i) * T + j] * (d_a[(b * T + i) * T + j] - dot);
        }
      vecf d_q(B * T * D, 0.0f), d_k(B * T * D, 0.0f);
      for (int64_t b = 0; b < B; ++b)
        for (int64_t i = 0; i < T; ++i)
          for (int64_t j = 0; j < T; ++j) {
            float ds = d_s[(b * T + i) * T + j] * scale;
            for (int64_t d = 0; d < D; ++d) {
              d_q[(b * T + i) * D + d] += ds * xs[(b * T + j) * D + d];
              d_k[(b * T + j) * D + d] += ds * xs[(b * T + i) * D + d];
            }
          }
      vecf dx = d_v;
      for (size_t i = 0; i < dx.size(); ++i) dx[i] += d_q[i] + d_k[i];
      add_side(st.x_at, dx);
      dy = dx;
    }
  }
  std::copy(dy.begin(), dy.end(), dx_out);
}

}  // extern "C"

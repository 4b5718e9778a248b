// ad.cu — exact rational reverse-mode differentiation with an explicit
// residual: the scalar lenses of the crate's src/ad.rs, on the host.
//
// An expression is a flat array of dop_expr_node (children by index), the
// C-ABI form of `ad::Expr` (src/ad.rs:49-59).  dop_ad_forward is `forward`
// (:76-129): it returns the value and a residual (tape) that stores only
// what the backward map reads — the two factors of every product, the branch
// a conditional took, nothing for sums, negations or projections.
// dop_ad_backward is `backward` (:131-176): the cotangent of every variable
// from the residual and the output cotangent.  dop_ad_stored_scalars is
// `stored_scalars` (:179-196).  Rationals stay reduced with a positive
// denominator (`Q::new`, :15-25); an i64 overflow is an error here, where the
// crate's release build would wrap.
#include <cstdint>
#include <cstdlib>
#include <vector>

#include "../../include/dop.h"
#include "common.cuh"

namespace dop {
int set_last_error(int code, const char* msg);

namespace ad {

struct Q {
  int64_t n = 0, d = 1;
};

int64_t gcd64(int64_t a, int64_t b) {
  while (b != 0) {
    const int64_t r = a % b;
    a = b;
    b = r;
  }
  return a < 1 ? 1 : a;
}

int64_t mul_checked(int64_t a, int64_t b) {
  int64_t r;
  if (__builtin_mul_overflow(a, b, &r)) throw Error(DOP_E_INVALID, "rational arithmetic overflows int64");
  return r;
}
int64_t add_checked(int64_t a, int64_t b) {
  int64_t r;
  if (__builtin_add_overflow(a, b, &r)) throw Error(DOP_E_INVALID, "rational arithmetic overflows int64");
  return r;
}

Q make(int64_t n, int64_t d) {
  DOP_REQUIRE(d != 0, "rational with zero denominator");
  if (d < 0) {
    DOP_REQUIRE(n != INT64_MIN && d != INT64_MIN, "rational arithmetic overflows int64");
    n = -n;
    d = -d;
  }
  DOP_REQUIRE(n != INT64_MIN, "rational arithmetic overflows int64");
  const int64_t g = gcd64(n < 0 ? -n : n, d);
  return Q{n / g, d / g};
}
Q add(Q a, Q b) { return make(add_checked(mul_checked(a.n, b.d), mul_checked(b.n, a.d)), mul_checked(a.d, b.d)); }
Q mul(Q a, Q b) { return make(mul_checked(a.n, b.n), mul_checked(a.d, b.d)); }
Q neg(Q a) { return make(-a.n, a.d); }
bool eq(Q a, Q b) { return a.n == b.n && a.d == b.d; }

// One residual node (`ad::Tape`, src/ad.rs:61-74); children by index.
struct TapeNode {
  int kind;          // DOP_EXPR_* of the expression node it was made from
  int64_t var = 0;   // Var
  Q x, y;            // Mul: the two factors
  int then_branch = 0;
  int64_t c0 = -1, c1 = -1;
};

struct Tape {
  std::vector<TapeNode> nodes;
  int64_t root = -1;
};

struct Ctx {
  const dop_expr_node* e;
  int64_t n;
};

const dop_expr_node& node(const Ctx& c, int64_t i) {
  DOP_REQUIRE(i >= 0 && i < c.n, "expression child index out of range");
  return c.e[i];
}

int64_t forward(const Ctx& c, int64_t i, const std::vector<Q>& env, Tape& t, Q& value, int depth) {
  DOP_REQUIRE(depth < 10000, "expression nests too deeply (or has a cycle)");
  const dop_expr_node& x = node(c, i);
  TapeNode tn;
  tn.kind = x.kind;
  switch (x.kind) {
    case DOP_EXPR_VAR:
      DOP_REQUIRE(x.var >= 0 && x.var < (int64_t)env.size(), "variable index out of range");
      value = env[x.var];
      tn.var = x.var;
      break;
    case DOP_EXPR_CONST:
      value = make(x.q.n, x.q.d);
      break;
    case DOP_EXPR_NEG: {
      Q v;
      tn.c0 = forward(c, x.a, env, t, v, depth + 1);
      value = neg(v);
      break;
    }
    case DOP_EXPR_ADD:
    case DOP_EXPR_MUL: {
      Q va, vb;
      tn.c0 = forward(c, x.a, env, t, va, depth + 1);
      tn.c1 = forward(c, x.b, env, t, vb, depth + 1);
      if (x.kind == DOP_EXPR_ADD) {
        value = add(va, vb);
      } else {
        value = mul(va, vb);
        tn.x = va;  // the factors, not the product
        tn.y = vb;
      }
      break;
    }
    case DOP_EXPR_LET: {  // let x = a in b, x at index 0 of b's environment
      Q vb;
      tn.c0 = forward(c, x.a, env, t, vb, depth + 1);
      std::vector<Q> ext;
      ext.reserve(env.size() + 1);
      ext.push_back(vb);
      ext.insert(ext.end(), env.begin(), env.end());
      tn.c1 = forward(c, x.b, ext, t, value, depth + 1);
      break;
    }
    case DOP_EXPR_IFEQ: {  // if a == b then c else d; only the taken branch is kept
      Q v1, v2;
      Tape scratch;  // the comparison's residuals are not kept
      forward(c, x.a, env, scratch, v1, depth + 1);
      forward(c, x.b, env, scratch, v2, depth + 1);
      tn.then_branch = eq(v1, v2) ? 1 : 0;
      tn.c0 = forward(c, tn.then_branch ? x.c : x.d, env, t, value, depth + 1);
      break;
    }
    default:
      throw Error(DOP_E_INVALID, "unknown expression node kind");
  }
  t.nodes.push_back(tn);
  return (int64_t)t.nodes.size() - 1;
}

void backward(const Ctx& c, int64_t i, const Tape& t, int64_t ti, Q cot, std::vector<Q>& acc,
              int depth) {
  DOP_REQUIRE(depth < 10000, "expression nests too deeply");
  const dop_expr_node& x = node(c, i);
  DOP_REQUIRE(ti >= 0 && ti < (int64_t)t.nodes.size(), "tape does not match expression");
  const TapeNode& tn = t.nodes[ti];
  DOP_REQUIRE(tn.kind == x.kind, "tape does not match expression");
  switch (x.kind) {
    case DOP_EXPR_VAR:
      DOP_REQUIRE(tn.var == x.var && x.var < (int64_t)acc.size(), "tape does not match expression");
      acc[x.var] = add(acc[x.var], cot);
      break;
    case DOP_EXPR_CONST:
      break;
    case DOP_EXPR_NEG:
      backward(c, x.a, t, tn.c0, neg(cot), acc, depth + 1);
      break;
    case DOP_EXPR_ADD:
      backward(c, x.a, t, tn.c0, cot, acc, depth + 1);
      backward(c, x.b, t, tn.c1, cot, acc, depth + 1);
      break;
    case DOP_EXPR_MUL:  // d(ab) = b da + a db from the stored factors
      backward(c, x.a, t, tn.c0, mul(cot, tn.y), acc, depth + 1);
      backward(c, x.b, t, tn.c1, mul(cot, tn.x), acc, depth + 1);
      break;
    case DOP_EXPR_LET: {
      std::vector<Q> body(acc.size() + 1);
      backward(c, x.b, t, tn.c1, cot, body, depth + 1);
      for (size_t v = 1; v < body.size(); ++v) acc[v - 1] = add(acc[v - 1], body[v]);
      backward(c, x.a, t, tn.c0, body[0], acc, depth + 1);
      break;
    }
    case DOP_EXPR_IFEQ:
      backward(c, tn.then_branch ? x.c : x.d, t, tn.c0, cot, acc, depth + 1);
      break;
    default:
      throw Error(DOP_E_INVALID, "unknown expression node kind");
  }
}

void stored(const Tape& t, int64_t ti, std::vector<Q>& out) {
  const TapeNode& tn = t.nodes[ti];
  if (tn.kind == DOP_EXPR_MUL) {
    out.push_back(tn.x);
    out.push_back(tn.y);
  }
  if (tn.c0 >= 0) stored(t, tn.c0, out);
  if (tn.c1 >= 0) stored(t, tn.c1, out);
}

}  // namespace ad
}  // namespace dop

struct dop_ad_tape {
  dop::ad::Tape t;
};

#define DOP_AD_GUARD(...)                                        \
  try {                                                          \
    __VA_ARGS__;                                                 \
    return DOP_OK;                                               \
  } catch (const dop::Error& e) {                                \
    return dop::set_last_error(e.code, e.what());                \
  } catch (const std::bad_alloc&) {                              \
    return dop::set_last_error(DOP_E_NOMEM, "host allocation failed"); \
  } catch (const std::exception& e) {                            \
    return dop::set_last_error(DOP_E_INVALID, e.what());         \
  }

extern "C" {

int dop_ad_forward(const dop_expr_node* nodes, int64_t n_nodes, int64_t root, const dop_q* env,
                   int64_t env_len, dop_q* value, dop_ad_tape** tape) {
  DOP_AD_GUARD({
    DOP_REQUIRE(nodes && value && tape && n_nodes > 0 && env_len >= 0 && (env || env_len == 0),
                "null pointer or empty expression");
    using namespace dop::ad;
    std::vector<Q> e(env_len);
    for (int64_t i = 0; i < env_len; ++i) e[i] = make(env[i].n, env[i].d);
    auto* t = new dop_ad_tape();
    try {
      Q v;
      t->t.root = forward(Ctx{nodes, n_nodes}, root, e, t->t, v, 0);
      value->n = v.n;
      value->d = v.d;
    } catch (...) {
      delete t;
      throw;
    }
    *tape = t;
  })
}

int dop_ad_backward(const dop_expr_node* nodes, int64_t n_nodes, int64_t root,
                    const dop_ad_tape* tape, dop_q cot, int64_t env_len, dop_q* cot_env) {
  DOP_AD_GUARD({
    DOP_REQUIRE(nodes && tape && cot_env && n_nodes > 0 && env_len >= 0, "null pointer");
    using namespace dop::ad;
    std::vector<Q> acc(env_len);
    backward(Ctx{nodes, n_nodes}, root, tape->t, tape->t.root, make(cot.n, cot.d), acc, 0);
    for (int64_t i = 0; i < env_len; ++i) cot_env[i] = dop_q{acc[i].n, acc[i].d};
  })
}

int dop_ad_stored_scalars(const dop_ad_tape* tape, dop_q* out, int64_t cap, int64_t* count) {
  DOP_AD_GUARD({
    DOP_REQUIRE(tape && count && (out || cap == 0), "null pointer");
    std::vector<dop::ad::Q> s;
    if (tape->t.root >= 0) dop::ad::stored(tape->t, tape->t.root, s);
    *count = (int64_t)s.size();
    DOP_REQUIRE((int64_t)s.size() <= cap || !out, "output capacity too small");
    for (size_t i = 0; i < s.size() && out; ++i) out[i] = dop_q{s[i].n, s[i].d};
  })
}

int dop_ad_tape_destroy(dop_ad_tape* tape) {
  delete tape;
  return DOP_OK;
}

}  // extern "C"

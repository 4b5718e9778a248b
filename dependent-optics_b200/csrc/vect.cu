// vect.cu — linear maps between finite-dimensional GF(2) vector spaces: the
// crate's src/vect.rs on the host.  A map is stored by the images of the
// basis vectors, each a u32 bitset (`Lin`, src/vect.rs:6-11), so domains have
// at most 32 dimensions and codomains at most 32.  `transpose` is the adjoint
// (the "put") of a linear map.  Dimension 0 has exactly one map, the zero map.
#include <cstdint>

#include "../../include/dop.h"
#include "common.cuh"

namespace dop {
int set_last_error(int code, const char* msg);

namespace vect {

void check(const dop_lin& f) {
  DOP_REQUIRE(f.dom <= 32 && f.cod <= 32, "GF(2) maps have at most 32 dimensions");
  const uint32_t mask = f.cod == 32 ? 0xffffffffu : ((1u << f.cod) - 1u);
  for (uint32_t j = 0; j < f.dom; ++j)
    DOP_REQUIRE((f.columns[j] & ~mask) == 0, "a column has bits outside the codomain");
}

// `Lin::apply_vec` (src/vect.rs:14-22): XOR of the columns selected by v.
uint32_t apply(const dop_lin& f, uint32_t v) {
  uint32_t acc = 0;
  for (uint32_t j = 0; j < f.dom; ++j)
    if ((v >> j) & 1u) acc ^= f.columns[j];
  return acc;
}

dop_lin blank(uint32_t dom, uint32_t cod) {
  dop_lin r{};
  r.dom = dom;
  r.cod = cod;
  return r;
}

}  // namespace vect
}  // namespace dop

#define DOP_VECT_GUARD(...)                                      \
  try {                                                          \
    __VA_ARGS__;                                                 \
    return DOP_OK;                                               \
  } catch (const dop::Error& e) {                                \
    return dop::set_last_error(e.code, e.what());                \
  } catch (const std::exception& e) {                            \
    return dop::set_last_error(DOP_E_INVALID, e.what());         \
  }

using dop::vect::apply;
using dop::vect::blank;
using dop::vect::check;

extern "C" {

uint32_t dop_lin_apply(const dop_lin* f, uint32_t v) { return f ? apply(*f, v) : 0u; }

int dop_lin_zero(uint32_t dom, uint32_t cod, dop_lin* out) {
  DOP_VECT_GUARD({
    DOP_REQUIRE(out && dom <= 32 && cod <= 32, "bad arguments");
    *out = blank(dom, cod);
  })
}

int dop_lin_identity(uint32_t n, dop_lin* out) {
  DOP_VECT_GUARD({
    DOP_REQUIRE(out && n <= 32, "bad arguments");
    *out = blank(n, n);
    for (uint32_t i = 0; i < n; ++i) out->columns[i] = 1u << i;
  })
}

// g after f (src/vect.rs:40-47): column j of the result is g applied to f's.
int dop_lin_compose(const dop_lin* g, const dop_lin* f, dop_lin* out) {
  DOP_VECT_GUARD({
    DOP_REQUIRE(g && f && out, "null pointer");
    check(*g);
    check(*f);
    DOP_REQUIRE(f->cod == g->dom, "linear composition needs f.cod == g.dom");
    dop_lin r = blank(f->dom, g->cod);
    for (uint32_t j = 0; j < f->dom; ++j) r.columns[j] = apply(*g, f->columns[j]);
    *out = r;
  })
}

// f + g over GF(2) (src/vect.rs:49-63).
int dop_lin_add(const dop_lin* f, const dop_lin* g, dop_lin* out) {
  DOP_VECT_GUARD({
    DOP_REQUIRE(g && f && out, "null pointer");
    check(*g);
    check(*f);
    DOP_REQUIRE(f->dom == g->dom && f->cod == g->cod, "added maps need equal shapes");
    dop_lin r = blank(f->dom, f->cod);
    for (uint32_t j = 0; j < f->dom; ++j) r.columns[j] = f->columns[j] ^ g->columns[j];
    *out = r;
  })
}

// The adjoint: bit i of column j becomes bit j of column i (src/vect.rs:65-79).
int dop_lin_transpose(const dop_lin* f, dop_lin* out) {
  DOP_VECT_GUARD({
    DOP_REQUIRE(f && out, "null pointer");
    check(*f);
    dop_lin r = blank(f->cod, f->dom);
    for (uint32_t j = 0; j < f->dom; ++j)
      for (uint32_t i = 0; i < f->cod; ++i)
        if ((f->columns[j] >> i) & 1u) r.columns[i] ^= 1u << j;
    *out = r;
  })
}

// Kronecker product, basis of A (x) B ordered a * dim_b + b (src/vect.rs:81-106).
int dop_lin_kronecker(const dop_lin* f, const dop_lin* g, dop_lin* out) {
  DOP_VECT_GUARD({
    DOP_REQUIRE(g && f && out, "null pointer");
    check(*g);
    check(*f);
    DOP_REQUIRE((uint64_t)f->dom * g->dom <= 32 && (uint64_t)f->cod * g->cod <= 32,
                "the Kronecker product exceeds 32 dimensions");
    dop_lin r = blank(f->dom * g->dom, f->cod * g->cod);
    for (uint32_t ja = 0; ja < f->dom; ++ja)
      for (uint32_t jb = 0; jb < g->dom; ++jb) {
        uint32_t image = 0;
        for (uint32_t ia = 0; ia < f->cod; ++ia) {
          if (!((f->columns[ja] >> ia) & 1u)) continue;
          for (uint32_t ib = 0; ib < g->cod; ++ib)
            if ((g->columns[jb] >> ib) & 1u) image ^= 1u << (ia * g->cod + ib);
        }
        r.columns[ja * g->dom + jb] = image;
      }
    *out = r;
  })
}

// Every map dom -> cod, in the order of the bit mask whose bit j*cod+i is
// bit i of column j (src/vect.rs:108-126).  With out == NULL only *count is
// written.
int dop_lin_all(uint32_t dom, uint32_t cod, dop_lin* out, int64_t cap, int64_t* count) {
  DOP_VECT_GUARD({
    DOP_REQUIRE(count && dom <= 32 && cod <= 32, "bad arguments");
    const uint64_t bits = (uint64_t)dom * cod;
    DOP_REQUIRE(bits <= 24, "more than 2^24 maps");
    const int64_t total = (int64_t)1 << bits;
    *count = total;
    if (!out) return DOP_OK;
    DOP_REQUIRE(cap >= total, "output capacity too small");
    for (int64_t mask = 0; mask < total; ++mask) {
      dop_lin r = blank(dom, cod);
      for (uint32_t j = 0; j < dom; ++j)
        for (uint32_t i = 0; i < cod; ++i)
          if ((mask >> (j * cod + i)) & 1) r.columns[j] |= 1u << i;
      out[mask] = r;
    }
  })
}

}  // extern "C"

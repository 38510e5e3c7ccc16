// nimq.cu -- reader of .nimq (NIMQ2) quantised state dicts held in host memory,
// and registration of their tensors as device-resident weights.
//
// Stream layout (quant.nim:411-448 loadQuantStateDict / readQuantTensor
// quant.nim:386-409; written by export_to_nimq.py:580-605 and
// quant.nim:365-384), all little-endian:
//   string magic "NIMQ2"                 (int32 length + bytes)
//   int32 arch[5]
//   int32 count
//   count x { string name;
//             uint8 kind; int32 ndims; int32 dims[ndims];
//             int32 n_scales; float32 scales[n_scales]; float32 zeros[n_scales];
//             int32 group_size; int32 exponent_bits; int32 mantissa_bits;
//             int32 data_len; uint8 data[data_len] }
// Parsing is host-only and needs no device; registration uploads the packed
// codes once (the reference copies them into a QuantTensor at load and then
// dequantises on the host at every forward, nimformer.nim:94-133).
#include <cstring>
#include <string>
#include <vector>

#include "nimf_internal.h"

namespace nimf {

namespace {

struct Reader {
  const uint8_t* buf;
  int64_t len;
  int64_t off = 0;
  bool take(void* dst, int64_t n) {
    if (n < 0 || off + n > len) return false;
    if (n) std::memcpy(dst, buf + off, (size_t)n);
    off += n;
    return true;
  }
  bool skip(int64_t n, const uint8_t** at) {
    if (n < 0 || off + n > len) return false;
    *at = buf + off;
    off += n;
    return true;
  }
  bool i32(int32_t* v) { return take(v, 4); }
};

int parse_header(Reader& r, int32_t arch[5], int64_t* count) {
  int32_t n;
  const uint8_t* magic;
  if (!r.i32(&n) || n != 5 || !r.skip(n, &magic) || std::memcmp(magic, "NIMQ2", 5) != 0)
    return set_error(NIMF_ERR_ARG, "not a NIMQ2 stream (quant.nim:351 magic)");
  int32_t a[5], c;
  if (!r.take(a, sizeof(a)) || !r.i32(&c) || c < 0)
    return set_error(NIMF_ERR_SHAPE, "NIMQ2 header truncated");
  if (arch) std::memcpy(arch, a, sizeof(a));
  *count = c;
  return NIMF_OK;
}

int parse_tensor(Reader& r, nimf_nimq_tensor* t) {
  std::memset(t, 0, sizeof(*t));
  int32_t nl, nd, ns, gs, eb, mb, dl;
  const uint8_t* p;
  uint8_t kind;
  if (!r.i32(&nl) || !r.skip(nl, &p)) return set_error(NIMF_ERR_SHAPE, "NIMQ2 record name truncated");
  t->name = reinterpret_cast<const char*>(p);
  t->name_len = nl;
  if (!r.take(&kind, 1) || !r.i32(&nd) || nd < 0 || nd > 8)
    return set_error(NIMF_ERR_SHAPE, "NIMQ2 record: bad dimension count");
  t->kind = kind;
  t->ndims = nd;
  for (int i = 0; i < nd; ++i) {
    int32_t d;
    if (!r.i32(&d) || d < 0) return set_error(NIMF_ERR_SHAPE, "NIMQ2 record: bad dimension");
    t->dims[i] = d;
  }
  if (!r.i32(&ns) || ns < 0) return set_error(NIMF_ERR_SHAPE, "NIMQ2 record: bad scale count");
  t->n_scales = ns;
  if (!r.skip((int64_t)ns * 4, &t->scales) || !r.skip((int64_t)ns * 4, &t->zeros))
    return set_error(NIMF_ERR_SHAPE, "NIMQ2 record: scales truncated");
  if (!r.i32(&gs) || !r.i32(&eb) || !r.i32(&mb) || !r.i32(&dl) || dl < 0)
    return set_error(NIMF_ERR_SHAPE, "NIMQ2 record: header truncated");
  t->group_size = gs;
  t->exponent_bits = eb;
  t->mantissa_bits = mb;
  if (!r.skip(dl, &t->data)) return set_error(NIMF_ERR_SHAPE, "NIMQ2 record: data truncated");
  t->data_len = dl;
  return NIMF_OK;
}

std::vector<float> floats(const uint8_t* p, int64_t n) {
  std::vector<float> v((size_t)n);
  if (n) std::memcpy(v.data(), p, (size_t)n * 4);
  return v;
}

}  // namespace

}  // namespace nimf

using namespace nimf;

extern "C" {

int nimf_nimq_parse(const uint8_t* buf, int64_t len, int32_t arch[5], int64_t* count) {
  if (!buf || len < 0 || !count) return set_error(NIMF_ERR_ARG, "NULL buffer or count");
  Reader r{buf, len};
  int64_t c;
  NIMF_TRY(parse_header(r, arch, &c));
  nimf_nimq_tensor t;
  for (int64_t i = 0; i < c; ++i) NIMF_TRY(parse_tensor(r, &t));
  *count = c;
  return NIMF_OK;
}

int nimf_nimq_get(const uint8_t* buf, int64_t len, int64_t index, nimf_nimq_tensor* out) {
  if (!buf || len < 0 || !out) return set_error(NIMF_ERR_ARG, "NULL buffer or out");
  Reader r{buf, len};
  int64_t c;
  NIMF_TRY(parse_header(r, nullptr, &c));
  if (index < 0 || index >= c)
    return set_error(NIMF_ERR_ARG, "tensor index %lld outside [0, %lld)", (long long)index, (long long)c);
  for (int64_t i = 0; i <= index; ++i) NIMF_TRY(parse_tensor(r, out));
  return NIMF_OK;
}

int nimf_nimq_register(const uint8_t* buf, int64_t len, int64_t index, int64_t row_begin,
                       int64_t row_end, nimf_weight_t* out) {
  nimf_nimq_tensor t;
  NIMF_TRY(nimf_nimq_get(buf, len, index, &t));
  if (!out) return set_error(NIMF_ERR_ARG, "out is NULL");
  if (t.ndims != 2)
    return set_error(NIMF_ERR_SHAPE, "NIMQ2 tensor %lld has %d dimensions; a weight is W[N][K]",
                     (long long)index, t.ndims);
  const int64_t n = t.dims[0], k = t.dims[1];
  const int64_t bpr = (k + 1) / 2;
  switch (t.kind) {
    case NIMF_KIND_F32: {
      // raw float32 W[N][K] -> beMatmul's b = W^T [K][N]
      if (t.data_len != n * k * 4) return set_error(NIMF_ERR_SHAPE, "raw tensor: %lld data bytes", (long long)t.data_len);
      if (row_begin != 0 || row_end != n)
        return set_error(NIMF_ERR_UNSUPPORTED, "raw fp32 tensors are registered whole");
      std::vector<float> w = floats(t.data, n * k), b((size_t)(n * k));
      for (int64_t r = 0; r < n; ++r)
        for (int64_t c = 0; c < k; ++c) b[(size_t)(c * n + r)] = w[(size_t)(r * k + c)];
      return nimf_weight_register_f32(b.data(), k, n, out);
    }
    case NIMF_KIND_INT8: {
      // dequantizeInt8 / the transposed int8 branch use scale[0] (quant.nim:63-67, 331-336)
      if (t.data_len != n * k || t.n_scales < 1)
        return set_error(NIMF_ERR_SHAPE, "int8 tensor: %lld data bytes, %lld scales",
                         (long long)t.data_len, (long long)t.n_scales);
      const std::vector<float> s = floats(t.scales, 1);
      return nimf_weight_register_i8(reinterpret_cast<const int8_t*>(t.data), s.data(), 1, n, k,
                                     row_begin, row_end, out);
    }
    case NIMF_KIND_INT4_SYM:
    case NIMF_KIND_INT4_ASYM: {
      // Rows of ceil(K/2) bytes as dequantizeTensorTransposed reads them
      // (quant.nim:270-330).  Per group (group_size > 0), per row (n_scales ==
      // N) or per tensor.  Symmetric codes become asymmetric ones exactly:
      // nibble ^ 8 with zero point 8 gives (nib' - 8) * sc = signed(nib) * sc.
      if (t.data_len != n * bpr) return set_error(NIMF_ERR_SHAPE, "int4 tensor: %lld data bytes", (long long)t.data_len);
      const bool sym = t.kind == NIMF_KIND_INT4_SYM;
      const std::vector<float> sc = floats(t.scales, t.n_scales), zp = floats(t.zeros, t.n_scales);
      int64_t gs = t.group_size, ngr;
      std::vector<float> s2, z2;
      if (!sym && gs > 0) {
        ngr = (k + gs - 1) / gs;
        if (t.n_scales != n * ngr) return set_error(NIMF_ERR_SHAPE, "int4 per-group tensor: %lld scales", (long long)t.n_scales);
        s2 = sc;
        z2 = zp;
      } else {
        if (t.n_scales < 1) return set_error(NIMF_ERR_SHAPE, "int4 tensor without scales");
        const bool per_row = !sym && t.n_scales > 1;
        if (per_row && t.n_scales != n) return set_error(NIMF_ERR_SHAPE, "int4 per-row tensor: %lld scales", (long long)t.n_scales);
        gs = 0;
        ngr = 1;
        s2.resize((size_t)n);
        z2.resize((size_t)n);
        for (int64_t r = 0; r < n; ++r) {
          s2[(size_t)r] = per_row ? sc[(size_t)r] : sc[0];
          z2[(size_t)r] = sym ? 8.0f : (per_row ? zp[(size_t)r] : zp[0]);
        }
      }
      const uint8_t* wq = t.data;
      std::vector<uint8_t> flip;
      if (sym) {
        flip.assign(t.data, t.data + t.data_len);
        for (auto& b : flip) b ^= 0x88;
        wq = flip.data();
      }
      return nimf_weight_register_q4g(wq, s2.data(), z2.data(), n, k, gs, ngr, row_begin, row_end, out);
    }
    case 4:  // fp8 e4m3, fp8 e5m2, custom, auto: CustomFloat codes (quant.nim:254)
    case 5:
    case NIMF_KIND_CUSTOM_FLOAT:
    case 7: {
      const int item = (1 + t.exponent_bits + t.mantissa_bits + 7) / 8;
      if (t.data_len != n * k * item) return set_error(NIMF_ERR_SHAPE, "CustomFloat tensor: %lld data bytes", (long long)t.data_len);
      return nimf_weight_register_cf(t.data, t.exponent_bits, t.mantissa_bits, nullptr, n, k,
                                     row_begin, row_end, out);
    }
  }
  return set_error(NIMF_ERR_UNSUPPORTED, "NIMQ2 tensor kind %d", t.kind);
}

}  // extern "C"

// The B200 target's compiler stand-in (include/hxb200_compiler.h): dispatch
// recognition, HMX-equivalent eligibility and strategy selection, compile-time
// tile plans, and serialisation of the executable.
//
// Eligibility follows the reference's rules for HMX contractions:
//   * analyzeSupportedContraction (ContractionStrategy.cpp:26-55): exactly
//     one M, N and K dimension, at most one batch dimension;
//   * hasHmxElementTypes (:138-150): one init, f16 inputs, f16 or f32
//     output;
//   * isHmxLowerableMatmul (:152-168): the output holds M before N;
//   * HexagonSpecializeHmxContractions.cpp:29-60: a linalg.generic that is
//     such a contraction is taken like the named matmul it specialises to;
//   * selectHmxStrategy (:170-213): batch tiled to 1 (one dispatch per batch
//     here), the compute tile chosen by the planner (here the B200 tile plan
//     from the baked sweep table or the cost model, hxb_plan_matmul_f16).
// Elementwise f16 -> f32 extensions feeding a contraction are folded into it
// (the f32 body of a fused dispatch that reads f16 tensors, as the
// specialisation pass describes). The B200 target also forms the int8-weight
// dispatch and the fused attention dispatch, which the reference compiles
// into HVX code (no int8 HMX path, ContractionStrategy.cpp:141; attention as
// separate dispatches, attention_layer.mlir:17-111).
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <cstdint>
#include <algorithm>
#include <functional>
#include <map>
#include <set>
#include <sstream>
#include <string>
#include <vector>

#include "hxb200_compiler.h"
#include "hxb200_hal.h"
#include "mlir_text.h"

namespace hxbc {
namespace {

constexpr char kMagic[4] = {'H', 'X', 'B', 'X'};
constexpr uint32_t kBlobVersion = 1;

enum StorageKind : uint32_t { kArg = 0, kResult = 1, kTransient = 2, kNone = 3 };

struct Binding {
  uint32_t kind = kNone;
  uint32_t index = 0;
  uint64_t offset = 0;
  uint64_t length = 0;
};

struct Dispatch {
  uint32_t ordinal = 0;
  std::vector<uint32_t> constants;
  std::vector<Binding> bindings;
};

struct Desc {
  int32_t elem = 0;
  std::vector<long long> dims;
};

struct CompiledFunc {
  std::string name;
  std::vector<Desc> args, results;
  std::vector<uint64_t> transients;
  std::vector<Dispatch> dispatches;
};

int elem_code(const std::string& e) {
  if (e == "f16") return HXB_ELEMENT_F16;
  if (e == "f32") return HXB_ELEMENT_F32;
  if (e == "i8") return HXB_ELEMENT_I8;
  return -1;
}

uint64_t elem_bytes(const std::string& e) {
  if (e == "f16" || e == "bf16") return 2;
  if (e == "f32" || e == "i32") return 4;
  if (e == "i8" || e == "i1") return 1;
  return 8;
}

uint64_t type_bytes(const TensorType& t) {
  uint64_t n = elem_bytes(t.elem);
  for (long long d : t.dims) n *= (uint64_t)d;
  return n;
}

uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}

// Parses the numeric text of a constant: decimal, or hex bits of the given
// float width.
bool constant_value(const std::string& text, const std::string& type, double* out) {
  if (text.empty()) return false;
  if (text.rfind("dense<", 0) == 0) {
    const std::string inner = text.substr(6, text.size() - 7);
    if (inner.find('[') != std::string::npos || inner.find(',') != std::string::npos) return false;
    return constant_value(inner, type, out);
  }
  if (text.size() > 2 && text[0] == '0' && (text[1] == 'x' || text[1] == 'X')) {
    const unsigned long long bits = strtoull(text.c_str() + 2, nullptr, 16);
    if (type == "f32") {
      const uint32_t b = (uint32_t)bits;
      float f;
      memcpy(&f, &b, 4);
      *out = f;
      return true;
    }
    if (type == "f64") {
      double d;
      memcpy(&d, &bits, 8);
      *out = d;
      return true;
    }
    return false;
  }
  char* end = nullptr;
  *out = strtod(text.c_str(), &end);
  return end && *end == '\0';
}

class FuncCompiler {
 public:
  FuncCompiler(const Module& m, const Func& f, const hxb_compiler_options_t& o,
               std::ostringstream& log)
      : m_(m), f_(f), opt_(o), log_(log) {}

  // false on a compile error (reported in the log)
  bool run(CompiledFunc* out);
  bool has_linalg() const {
    for (const Op& op : f_.ops)
      if (op.name.rfind("linalg.", 0) == 0) return true;
    return false;
  }

 private:
  const Module& m_;
  const Func& f_;
  const hxb_compiler_options_t& opt_;
  std::ostringstream& log_;

  struct Def {
    int op = -1;   // index into f_.ops, -1 for a function argument
    int arg = -1;  // function argument index
  };
  std::map<std::string, Def> defs_;
  std::map<std::string, std::string> types_;
  std::map<std::string, int> uses_;
  std::set<int> consumed_;
  // values whose storage is fixed: function arguments (by import) and results
  std::map<std::string, Binding> storage_;
  CompiledFunc* out_ = nullptr;

  // -------------------------------------------------------------- helpers
  void err(const Op& op, const std::string& msg) {
    log_ << "error @" << f_.name << " line " << op.line << ": " << op.name << ": " << msg << "\n";
  }
  void note(const char* kind, const Op& op, const std::string& msg) {
    log_ << kind << " @" << f_.name << " line " << op.line << ": " << op.name << ": " << msg
         << "\n";
  }
  const Op* def_op(const std::string& v, int* index = nullptr) const {
    auto it = defs_.find(v);
    if (it == defs_.end() || it->second.op < 0) return nullptr;
    if (index) *index = it->second.op;
    return &f_.ops[it->second.op];
  }
  TensorType type_of(const std::string& v) const {
    auto it = types_.find(v);
    return it == types_.end() ? TensorType{} : parse_type(it->second);
  }

  AffineMap map_of(const Tok& t) const {
    if (t.k == Tok::kHash) {
      auto it = m_.aliases.find(t.s);
      return it == m_.aliases.end() ? AffineMap{} : parse_affine_map(it->second);
    }
    return parse_affine_map(t.s);
  }
  std::vector<AffineMap> maps_of(const Op& op) const {
    std::vector<AffineMap> out;
    for (const Tok& t : op_attr(op, "indexing_maps"))
      if (t.k == Tok::kHash || t.k == Tok::kAngle) out.push_back(map_of(t));
    return out;
  }
  std::vector<std::string> iterators_of(const Op& op) const {
    std::vector<std::string> out;
    for (const Tok& t : op_attr(op, "iterator_types"))
      if (t.k == Tok::kStr) out.push_back(t.s);
    return out;
  }
  static bool identity(const AffineMap& m) {
    if (!m.ok || (int)m.results.size() != m.num_dims) return false;
    for (int i = 0; i < m.num_dims; ++i)
      if (m.results[i] != i) return false;
    return true;
  }

  // An elementwise linalg.generic: one output, identity maps on every operand
  // of the output's rank, all iterators parallel.
  bool elementwise(const Op& op) const {
    if (op.name != "linalg.generic" || op.region.size() != 1) return false;
    for (const std::string& it : iterators_of(op))
      if (it != "parallel") return false;
    for (const AffineMap& m : maps_of(op))
      if (!identity(m)) return false;
    return true;
  }

  // The body ops of a generic, without the terminator.
  static const std::vector<Op>& body(const Op& op) { return op.region[0].ops; }
  static const Op& yield(const Op& op) { return op.region[0].ops.back(); }

  // If `v` is produced by an elementwise generic whose body is a single
  // `cast` (e.g. arith.extf) of its input, returns that input; else "".
  std::string unary_source(const std::string& v, const char* cast, int* index = nullptr) const {
    int idx = -1;
    const Op* op = def_op(v, &idx);
    if (!op || !elementwise(*op) || body(*op).size() != 2) return "";
    std::vector<std::string> ins, ins_t;
    if (!op_group(*op, "ins", &ins, &ins_t) || ins.size() != 1) return "";
    const Op& b = body(*op)[0];
    const auto& blk = op->region[0];
    if (b.name != cast || op_operands(b).size() != 1 || op_operands(b)[0] != blk.args[0])
      return "";
    if (op_operands(yield(*op)).size() != 1 || op_operands(yield(*op))[0] != b.results[0])
      return "";
    if (index) *index = idx;
    return ins[0];
  }

  // The f16 tensor behind an f32 operand: folds an elementwise f16 -> f32
  // extension (marking it consumed when `consume`).
  std::string f16_source(const std::string& v, bool consume) {
    const TensorType t = type_of(v);
    if (t.ok && t.elem == "f16") return v;
    int idx = -1;
    const std::string src = unary_source(v, "arith.extf", &idx);
    if (!src.empty() && type_of(src).elem == "f16") {
      if (consume) consumed_.insert(idx);
      return src;
    }
    return "";
  }

  // Zero-filled tensor (linalg.fill of the constant 0): true, and marks the
  // fill consumed when `consume`.
  bool zero_fill(const std::string& v, bool consume) {
    int idx = -1;
    const Op* op = def_op(v, &idx);
    if (!op || op->name != "linalg.fill") return false;
    std::vector<std::string> ins, ins_t;
    if (!op_group(*op, "ins", &ins, &ins_t) || ins.size() != 1) return false;
    const Op* c = def_op(ins[0]);
    double x = 1.0;
    if (!c || c->name != "arith.constant" || !ins_t.size() ||
        !constant_value(op_constant_text(*c), ins_t[0], &x) || x != 0.0)
      return false;
    if (consume) consumed_.insert(idx);
    return true;
  }

  bool fill_value(const std::string& v, double* x, int* index) {
    const Op* op = def_op(v, index);
    if (!op || op->name != "linalg.fill") return false;
    std::vector<std::string> ins, ins_t;
    if (!op_group(*op, "ins", &ins, &ins_t) || ins.size() != 1) return false;
    const Op* c = def_op(ins[0]);
    return c && c->name == "arith.constant" && !ins_t.empty() &&
           constant_value(op_constant_text(*c), ins_t[0], x);
  }

  // Storage of a value a dispatch reads: a function argument or result, or
  // the transient buffer another dispatch wrote.
  Binding storage_of(const std::string& v) {
    auto it = storage_.find(v);
    if (it != storage_.end()) return it->second;
    return Binding{};
  }

  // Storage of a value a dispatch writes: its result slot if it is returned,
  // else a new transient buffer.
  Binding output_storage(const std::string& v) {
    auto it = storage_.find(v);
    if (it != storage_.end()) return it->second;
    Binding b;
    b.kind = kTransient;
    b.index = (uint32_t)out_->transients.size();
    b.length = type_bytes(type_of(v));
    out_->transients.push_back(b.length);
    storage_[v] = b;
    return b;
  }

  Binding slice(Binding b, uint64_t offset, uint64_t length) {
    b.offset += offset;
    b.length = length;
    return b;
  }

  // --------------------------------------------------------------- patterns
  bool try_attention(int i);
  bool try_w8(int i);
  bool try_contraction(int i);

  // One M, N, K and at most one batch dimension of a contraction given its
  // operand maps (lhs, rhs, out) and iterator types.
  struct Dims {
    int m = -1, n = -1, k = -1, b = -1;
  };
  static bool contraction_dims(const AffineMap& a, const AffineMap& bm, const AffineMap& c,
                               const std::vector<std::string>& it, Dims* d, std::string* why) {
    const int nd = a.num_dims;
    std::vector<int> ms, ns, ks, bs;
    auto has = [](const AffineMap& m, int dim) {
      for (int r : m.results)
        if (r == dim) return true;
      return false;
    };
    for (int x = 0; x < nd; ++x) {
      const bool ina = has(a, x), inb = has(bm, x), inc = has(c, x);
      const bool red = x < (int)it.size() && it[x] == "reduction";
      if (ina && inb && inc && !red)
        bs.push_back(x);
      else if (ina && !inb && inc && !red)
        ms.push_back(x);
      else if (!ina && inb && inc && !red)
        ns.push_back(x);
      else if (ina && inb && !inc && red)
        ks.push_back(x);
      else {
        *why = "dimension d" + std::to_string(x) + " is not a batch, M, N or K dimension";
        return false;
      }
    }
    if (ms.size() != 1 || ns.size() != 1 || ks.size() != 1 || bs.size() > 1) {
      *why = "needs exactly one M, N and K dimension and at most one batch dimension "
             "(ContractionStrategy.cpp:26-55)";
      return false;
    }
    d->m = ms[0];
    d->n = ns[0];
    d->k = ks[0];
    d->b = bs.empty() ? -1 : bs[0];
    return true;
  }
  static int pos(const AffineMap& m, int dim) {
    for (size_t i = 0; i < m.results.size(); ++i)
      if (m.results[i] == dim) return (int)i;
    return -1;
  }

  bool has_bindings() const;
  bool program_form(CompiledFunc* out);
  bool dispatch_form(CompiledFunc* out);

  bool emit_matmul(const Op& op, const std::string& a, const std::string& b,
                   const std::string& init, const std::string& res, long long batch,
                   long long M, long long N, long long K, bool transpose_b, bool zero_init);
};

bool FuncCompiler::emit_matmul(const Op& op, const std::string& a, const std::string& b,
                               const std::string& init, const std::string& res,
                               long long batch, long long M, long long N, long long K,
                               bool transpose_b, bool zero_init) {
  const TensorType rt = type_of(res);
  const bool f32 = rt.elem == "f32";
  const Binding ab = storage_of(a), bb = storage_of(b);
  if (ab.kind == kNone || bb.kind == kNone) {
    err(op, "an operand is neither a function argument nor a dispatch result");
    return false;
  }
  Binding ib;
  if (!zero_init) {
    ib = storage_of(init);
    if (ib.kind == kNone) {
      err(op, "the init is neither zero nor a function argument or dispatch result");
      return false;
    }
  }
  const Binding cb = output_storage(res);
  int bn = 0, gm = 0, sk = 1, pair = 1;
  if (hxb_plan_matmul_f16(M, N, K, transpose_b ? 1 : 0, opt_.num_sms ? opt_.num_sms : 148, &bn,
                          &gm, &sk, &pair) != HXB_OK) {
    err(op, "no tile plan for this shape");
    return false;
  }
  const uint64_t esz = f32 ? 4 : 2;
  for (long long bi = 0; bi < batch; ++bi) {
    Dispatch d;
    d.ordinal = HXB_EXPORT_MATMUL_F16;
    d.constants = {(uint32_t)M, (uint32_t)N, (uint32_t)K,
                   (transpose_b ? 1u : 0u) | (f32 ? 2u : 0u), (uint32_t)bn, (uint32_t)gm,
                   (uint32_t)sk, (uint32_t)pair};
    d.bindings.push_back(slice(ab, (uint64_t)bi * M * K * 2, (uint64_t)M * K * 2));
    d.bindings.push_back(slice(bb, (uint64_t)bi * K * N * 2, (uint64_t)K * N * 2));
    d.bindings.push_back(slice(cb, (uint64_t)bi * M * N * esz, (uint64_t)M * N * esz));
    if (!zero_init) d.bindings.push_back(slice(ib, (uint64_t)bi * M * N * esz, (uint64_t)M * N * esz));
    out_->dispatches.push_back(std::move(d));
  }
  std::ostringstream s;
  s << "matmul_f16 dispatch" << (batch > 1 ? "es" : "") << ": " << (batch > 1 ? std::to_string(batch) + " x " : "")
    << M << "x" << N << "x" << K << (transpose_b ? " (rhs transposed)" : "")
    << (f32 ? ", f32 out" : ", f16 out") << (zero_init ? "" : ", init added")
    << "; tile plan block_n " << bn << ", group_m " << gm << ", split_k " << sk
    << ", cta_pair " << pair;
  note("accept", op, s.str());
  return true;
}

bool FuncCompiler::try_contraction(int i) {
  const Op& op = f_.ops[i];
  std::vector<std::string> ins, ins_t, outs, outs_t;
  if (!op_group(op, "ins", &ins, &ins_t) || !op_group(op, "outs", &outs, &outs_t)) return false;
  AffineMap am, bmap, cm;
  std::vector<std::string> it;
  const std::string& n = op.name;
  const bool named = n == "linalg.matmul" || n == "linalg.batch_matmul" ||
                     n == "linalg.matmul_transpose_b" || n == "linalg.batch_matmul_transpose_b";
  if (named) {
    const bool batch = n.find("batch") != std::string::npos;
    const bool tb = n.find("transpose_b") != std::string::npos;
    const char* txt;
    if (!batch)
      txt = tb ? "(m, n, k) -> (m, k)|(m, n, k) -> (n, k)|(m, n, k) -> (m, n)"
               : "(m, n, k) -> (m, k)|(m, n, k) -> (k, n)|(m, n, k) -> (m, n)";
    else
      txt = tb ? "(b, m, n, k) -> (b, m, k)|(b, m, n, k) -> (b, n, k)|(b, m, n, k) -> (b, m, n)"
               : "(b, m, n, k) -> (b, m, k)|(b, m, n, k) -> (b, k, n)|(b, m, n, k) -> (b, m, n)";
    std::string s(txt);
    const size_t p1 = s.find('|'), p2 = s.find('|', p1 + 1);
    am = parse_affine_map(s.substr(0, p1));
    bmap = parse_affine_map(s.substr(p1 + 1, p2 - p1 - 1));
    cm = parse_affine_map(s.substr(p2 + 1));
    it.assign(am.num_dims, "parallel");
    it.back() = "reduction";
  } else if (n == "linalg.generic") {
    const auto maps = maps_of(op);
    it = iterators_of(op);
    bool red = false;
    for (const auto& x : it) red |= x == "reduction";
    if (!red || ins.size() != 2 || outs.size() != 1 || maps.size() != 3) return false;
    // body: acc + a * b (each factor possibly extended to f32)
    const auto& blk = op.region[0];
    const auto& bops = body(op);
    if (bops.size() < 3 || blk.args.size() != 3) return false;
    const Op& y = bops.back();
    if (y.name != "linalg.yield" || op_operands(y).size() != 1) return false;
    std::map<std::string, const Op*> by;
    for (const Op& b : bops)
      for (const auto& r : b.results) by[r] = &b;
    auto root = [&](std::string v) {
      while (by.count(v) && by[v]->name == "arith.extf") v = op_operands(*by[v])[0];
      return v;
    };
    const Op* add = by.count(op_operands(y)[0]) ? by[op_operands(y)[0]] : nullptr;
    if (!add || add->name != "arith.addf" || op_operands(*add).size() != 2) return false;
    auto ao = op_operands(*add);
    std::string prod = ao[0] == blk.args[2] ? ao[1] : (ao[1] == blk.args[2] ? ao[0] : "");
    if (prod.empty() || !by.count(prod) || by[prod]->name != "arith.mulf") return false;
    auto mo = op_operands(*by[prod]);
    if (mo.size() != 2) return false;
    std::set<std::string> f{root(mo[0]), root(mo[1])};
    if (f != std::set<std::string>{blk.args[0], blk.args[1]}) return false;
    am = maps[0];
    bmap = maps[1];
    cm = maps[2];
  } else {
    return false;
  }
  if (!opt_.enable_matmul) {
    note("reject", op, "matmul dispatches are disabled");
    return false;
  }
  if (!am.ok || !bmap.ok || !cm.ok) {
    err(op, "indexing maps are not projected permutations");
    return false;
  }
  Dims d;
  std::string why;
  if (!contraction_dims(am, bmap, cm, it, &d, &why)) {
    err(op, "not an HMX-shaped contraction: " + why);
    return false;
  }
  // hasHmxElementTypes: f16 inputs (after folding f16 -> f32 extensions),
  // one f16 or f32 init
  const std::string a = f16_source(ins[0], false), b = f16_source(ins[1], false);
  const TensorType ct = type_of(outs[0]);
  if (a.empty() || b.empty() || !(ct.elem == "f16" || ct.elem == "f32")) {
    err(op, "element types are not f16 inputs with an f16 or f32 init "
            "(hasHmxElementTypes, ContractionStrategy.cpp:138-150)");
    return false;
  }
  // isHmxLowerableMatmul: M before N in the output; the B200 kernel also
  // wants the lhs K-major (A[..., M, K])
  if (pos(cm, d.m) > pos(cm, d.n)) {
    err(op, "output holds N before M (isHmxLowerableMatmul, ContractionStrategy.cpp:152-168)");
    return false;
  }
  if (pos(am, d.m) > pos(am, d.k)) {
    err(op, "lhs holds K before M: no B200 dispatch for a transposed lhs");
    return false;
  }
  if (d.b >= 0 && (pos(am, d.b) != 0 || pos(bmap, d.b) != 0 || pos(cm, d.b) != 0)) {
    err(op, "the batch dimension must be outermost in every operand");
    return false;
  }
  const bool tb = pos(bmap, d.n) < pos(bmap, d.k);
  const TensorType at = type_of(a), bt = type_of(b);
  if (!at.ok || !bt.ok || !ct.ok) {
    err(op, "operand types are not static tensors");
    return false;
  }
  const long long M = ct.dims[pos(cm, d.m)], N = ct.dims[pos(cm, d.n)],
                  K = at.dims[pos(am, d.k)];
  const long long B = d.b >= 0 ? ct.dims[pos(cm, d.b)] : 1;
  if (M < 1 || N < 1 || K < 1 || M > 0x7fffffff || N > 0x7fffffff || K > 0x7fffffff) {
    err(op, "extents out of range");
    return false;
  }
  f16_source(ins[0], true);
  f16_source(ins[1], true);
  const bool zero = zero_fill(outs[0], true);
  consumed_.insert(i);
  return emit_matmul(op, a, b, outs[0], op.results[0], B, M, N, K, tb, zero);
}

bool FuncCompiler::try_w8(int i) {
  const Op& op = f_.ops[i];
  if (op.name != "linalg.generic" || op.region.size() != 1) return false;
  std::vector<std::string> ins, ins_t, outs, outs_t;
  if (!op_group(op, "ins", &ins, &ins_t) || !op_group(op, "outs", &outs, &outs_t)) return false;
  if (ins.size() != 3 || outs.size() != 1) return false;
  const TensorType at = type_of(ins[0]), wt = type_of(ins[1]), st = type_of(ins[2]),
                   ct = type_of(outs[0]);
  if (at.elem != "f16" || wt.elem != "i8" || st.elem != "f16" || ct.elem != "f32") return false;
  const auto maps = maps_of(op);
  const auto it = iterators_of(op);
  if (maps.size() != 4) return false;
  // body: acc + extf(a) * (sitofp(w) * extf(s)), factors in any order
  const auto& blk = op.region[0];
  std::map<std::string, const Op*> by;
  for (const Op& b : body(op))
    for (const auto& r : b.results) by[r] = &b;
  const Op& y = yield(op);
  if (op_operands(y).size() != 1 || !by.count(op_operands(y)[0])) return false;
  const Op* add = by[op_operands(y)[0]];
  if (add->name != "arith.addf") return false;
  std::vector<std::string> leaves;
  std::function<bool(const std::string&)> walk = [&](const std::string& v) -> bool {
    if (!by.count(v)) return false;
    const Op* o = by[v];
    if (o->name == "arith.mulf") {
      const auto x = op_operands(*o);
      return x.size() == 2 && walk(x[0]) && walk(x[1]);
    }
    if (o->name == "arith.extf" || o->name == "arith.sitofp") {
      leaves.push_back(o->name + ":" + op_operands(*o)[0]);
      return true;
    }
    return false;
  };
  const auto ao = op_operands(*add);
  if (ao.size() != 2) return false;
  const std::string prod = ao[0] == blk.args[3] ? ao[1] : (ao[1] == blk.args[3] ? ao[0] : "");
  if (prod.empty() || !walk(prod)) return false;
  std::multiset<std::string> want{"arith.extf:" + blk.args[0], "arith.sitofp:" + blk.args[1],
                                  "arith.extf:" + blk.args[2]};
  if (std::multiset<std::string>(leaves.begin(), leaves.end()) != want) return false;
  if (!opt_.enable_w8a16) {
    note("reject", op, "int8-weight dispatches are disabled");
    return false;
  }
  // A[m, k], W[k, n], scale[n] -> C[m, n]
  const AffineMap &ma = maps[0], &mw = maps[1], &ms = maps[2], &mc = maps[3];
  if (!ma.ok || !mw.ok || !ms.ok || !mc.ok || ma.results.size() != 2 || mw.results.size() != 2 ||
      ms.results.size() != 1 || mc.results.size() != 2) {
    err(op, "int8-weight contraction maps are not A[m,k], W[k,n], scale[n] -> C[m,n]");
    return false;
  }
  const int m = mc.results[0], n = mc.results[1], k = ma.results[1];
  if (ma.results[0] != m || mw.results[0] != k || mw.results[1] != n || ms.results[0] != n ||
      k < 0 || k >= (int)it.size() || it[k] != "reduction") {
    err(op, "int8-weight contraction maps are not A[m,k], W[k,n], scale[n] -> C[m,n]");
    return false;
  }
  if (!zero_fill(outs[0], false)) {
    err(op, "the int8-weight contraction must accumulate into a zero fill");
    return false;
  }
  // its f32 result must be truncated to f16 by the only user (the export
  // writes f16 with one rounding)
  int trunc_idx = -1;
  std::string trunc_res;
  for (int j = i + 1; j < (int)f_.ops.size(); ++j) {
    int idx = -1;
    for (const auto& r : f_.ops[j].results)
      if (unary_source(r, "arith.truncf", &idx) == op.results[0]) {
        trunc_idx = idx;
        trunc_res = r;
      }
    if (trunc_idx >= 0) break;
  }
  if (trunc_idx < 0 || uses_[op.results[0]] != 1 || type_of(trunc_res).elem != "f16") {
    err(op, "the int8-weight contraction's f32 result must feed only an f16 truncation");
    return false;
  }
  const long long M = ct.dims[0], N = ct.dims[1], K = at.dims[1];
  const Binding ab = storage_of(ins[0]), wb = storage_of(ins[1]), sb = storage_of(ins[2]);
  if (ab.kind == kNone || wb.kind == kNone || sb.kind == kNone) {
    err(op, "an operand is neither a function argument nor a dispatch result");
    return false;
  }
  zero_fill(outs[0], true);
  consumed_.insert(i);
  consumed_.insert(trunc_idx);
  const Binding cb = output_storage(trunc_res);
  Dispatch d;
  d.ordinal = HXB_EXPORT_MATMUL_W8A16;
  d.constants = {(uint32_t)M, (uint32_t)N, (uint32_t)K};
  d.bindings = {slice(ab, 0, (uint64_t)M * K * 2), slice(wb, 0, (uint64_t)K * N),
                slice(sb, 0, (uint64_t)N * 2), slice(cb, 0, (uint64_t)M * N * 2)};
  out_->dispatches.push_back(std::move(d));
  std::ostringstream s;
  s << "matmul_w8a16 dispatch: " << M << "x" << N << "x" << K
    << " (int8 weights, per-channel f16 scale, f16 out; truncf folded)";
  note("accept", op, s.str());
  return true;
}

bool FuncCompiler::try_attention(int i) {
  // root: O16 = truncf(batch_matmul(P, extf(V)) into zeros)
  const Op& root = f_.ops[i];
  const std::string o32 = unary_source(root.results.empty() ? "" : root.results[0], "arith.truncf");
  if (o32.empty()) return false;
  std::vector<int> chain;
  int idx = -1;
  auto def = [&](const std::string& v, const char* name) -> const Op* {
    int k = -1;
    const Op* o = def_op(v, &k);
    if (!o || o->name != name) return nullptr;
    idx = k;
    return o;
  };
  std::vector<std::string> ins, ins_t, outs, outs_t;
  const Op* pv = def(o32, "linalg.batch_matmul");
  if (!pv) return false;
  chain.push_back(idx);
  op_group(*pv, "ins", &ins, &ins_t);
  op_group(*pv, "outs", &outs, &outs_t);
  if (ins.size() != 2 || !zero_fill(outs[0], false)) return false;
  const std::string P = ins[0], V = f16_source(ins[1], false);
  if (V.empty()) return false;
  // P = select(mask, zeros, probs)
  const Op* sel = def(P, "linalg.generic");
  if (!sel || body(*sel).size() != 2 || body(*sel)[0].name != "arith.select") return false;
  chain.push_back(idx);
  op_group(*sel, "ins", &ins, &ins_t);
  if (ins.size() != 3) return false;
  const std::string mask = ins[0], probs = ins[2];
  // probs = E / sum(E)
  const Op* div = def(probs, "linalg.generic");
  if (!div || body(*div).size() != 2 || body(*div)[0].name != "arith.divf") return false;
  chain.push_back(idx);
  op_group(*div, "ins", &ins, &ins_t);
  if (ins.size() != 2) return false;
  const std::string E = ins[0], SUM = ins[1];
  const Op* sum = def(SUM, "linalg.generic");
  if (!sum || body(*sum).size() != 2 || body(*sum)[0].name != "arith.addf") return false;
  chain.push_back(idx);
  op_group(*sum, "ins", &ins, &ins_t);
  op_group(*sum, "outs", &outs, &outs_t);
  if (ins.size() != 1 || ins[0] != E || !zero_fill(outs[0], false)) return false;
  const std::string sum_init = outs[0];
  // E = exp(S - max(S))
  const Op* ex = def(E, "linalg.generic");
  if (!ex || body(*ex).size() != 2 || body(*ex)[0].name != "math.exp") return false;
  chain.push_back(idx);
  op_group(*ex, "ins", &ins, &ins_t);
  const Op* sub = def(ins.size() == 1 ? ins[0] : "", "linalg.generic");
  if (!sub || body(*sub).size() != 2 || body(*sub)[0].name != "arith.subf") return false;
  chain.push_back(idx);
  op_group(*sub, "ins", &ins, &ins_t);
  if (ins.size() != 2) return false;
  const std::string S = ins[0];
  const Op* exp_shape = def(ins[1], "tensor.expand_shape");
  if (!exp_shape) return false;
  chain.push_back(idx);
  std::string mx = op_operands(*exp_shape).empty() ? "" : op_operands(*exp_shape)[0];
  const std::string mx_base = mx.substr(0, mx.find('#'));
  const Op* maxr = nullptr;
  {
    int k = -1;
    maxr = def_op(mx, &k);
    if (!maxr || maxr->name != "linalg.generic") return false;
    bool has_max = false;
    for (const Op& b : body(*maxr)) has_max |= b.name == "arith.maximumf";
    op_group(*maxr, "ins", &ins, &ins_t);
    if (!has_max || ins.size() != 1 || ins[0] != S) return false;
    chain.push_back(k);
    std::vector<std::string> mo, mot;
    op_group(*maxr, "outs", &mo, &mot);
    double v = 0;
    int fi = -1;
    for (const auto& o : mo) {
      if (fill_value(o, &v, &fi)) chain.push_back(fi);
    }
  }
  // S = batch_matmul(Q * s, transpose(K) * s)
  const Op* qk = def(S, "linalg.batch_matmul");
  if (!qk) return false;
  chain.push_back(idx);
  op_group(*qk, "ins", &ins, &ins_t);
  op_group(*qk, "outs", &outs, &outs_t);
  if (ins.size() != 2 || !zero_fill(outs[0], false)) return false;
  const std::string qk_init = outs[0];
  auto scaled = [&](const std::string& v, std::string* src, double* s) -> bool {
    const Op* g = def(v, "linalg.generic");
    if (!g || body(*g).size() < 2) return false;
    const int gi = idx;
    std::vector<std::string> gi_ins, gi_t;
    op_group(*g, "ins", &gi_ins, &gi_t);
    if (gi_ins.size() != 1) return false;
    // body: [c = truncf(f64 const)]; mulf(in, c); yield
    const Op* mul = nullptr;
    std::string cval;
    for (const Op& b : body(*g)) {
      if (b.name == "arith.mulf") mul = &b;
    }
    if (!mul) return false;
    auto mo = op_operands(*mul);
    if (mo.size() != 2) return false;
    const std::string c = mo[0] == g->region[0].args[0] ? mo[1] : mo[0];
    // the scale: a constant, possibly truncated from f64 in the body
    std::string cname = c;
    bool trunc = false;
    for (const Op& b : body(*g))
      if (!b.results.empty() && b.results[0] == c && b.name == "arith.truncf") {
        cname = op_operands(b)[0];
        trunc = true;
      }
    const Op* cst = def_op(cname);
    if (!cst || cst->name != "arith.constant") return false;
    const auto ct = op_result_types(*cst);
    if (ct.empty() || !constant_value(op_constant_text(*cst), ct[0], s)) return false;
    if (trunc || ct[0] == "f32") *s = (double)(float)*s;  // the f32 factor the body applies
    *src = gi_ins[0];
    chain.push_back(gi);
    return true;
  };
  std::string qsrc, ksrc;
  double sq = 0, sk = 0;
  if (!scaled(ins[0], &qsrc, &sq) || !scaled(ins[1], &ksrc, &sk)) return false;
  const std::string Q = f16_source(qsrc, false);
  const Op* tr = def(ksrc, "linalg.transpose");
  if (!tr || Q.empty()) return false;
  chain.push_back(idx);
  std::vector<std::string> tins, tins_t;
  op_group(*tr, "ins", &tins, &tins_t);
  std::string perm;
  for (const Tok& t : op_attr(*tr, "permutation")) perm += t.s;
  if (tins.size() != 1 || perm != "[0,2,1]") return false;
  const std::string Kt = f16_source(tins[0], false);
  if (Kt.empty()) return false;
  // mask: and-reduction of (S == -inf) -> rows that see no key give 0
  const Op* mred = def(mask, "linalg.generic");
  if (!mred) return false;
  chain.push_back(idx);
  {
    std::vector<std::string> mi, mit, mo, mot;
    op_group(*mred, "ins", &mi, &mit);
    op_group(*mred, "outs", &mo, &mot);
    double v;
    int fi = -1;
    for (const auto& o : mo)
      if (fill_value(o, &v, &fi)) chain.push_back(fi);
    const Op* cmp = def(mi.size() == 1 ? mi[0] : "", "linalg.generic");
    if (!cmp) return false;
    chain.push_back(idx);
    bool has_cmp = false;
    for (const Op& b : body(*cmp)) has_cmp |= b.name == "arith.cmpf";
    op_group(*cmp, "ins", &mi, &mit);
    if (!has_cmp || mi.size() != 1 || mi[0] != S) return false;
  }
  if (!opt_.enable_attention) {
    note("reject", root, "attention dispatches are disabled");
    return false;
  }
  const TensorType qt = type_of(Q), kt = type_of(Kt), vt = type_of(V), ot = type_of(root.results[0]);
  if (qt.dims.size() != 3 || kt.dims.size() != 3 || vt.dims.size() != 3 || ot.elem != "f16") {
    err(root, "attention operands must be [batch*heads, seq, head_dim] f16");
    return false;
  }
  const long long BH = qt.dims[0], Sq = qt.dims[1], D = qt.dims[2], Skv = kt.dims[1];
  if (D != 64 && D != 128) {
    err(root, "attention head dim must be 64 or 128");
    return false;
  }
  const Binding qb = storage_of(Q), kb = storage_of(Kt), vb = storage_of(V);
  if (qb.kind == kNone || kb.kind == kNone || vb.kind == kNone) {
    err(root, "Q, K and V must be function arguments or dispatch results");
    return false;
  }
  // consume the chain and its f16 -> f32 extensions and zero fills
  for (int c : chain) consumed_.insert(c);
  consumed_.insert(i);
  f16_source(qsrc, true);
  f16_source(tins[0], true);
  f16_source(ins.size() ? ins[1] : "", false);
  {
    std::vector<std::string> pvins, pvt;
    op_group(*pv, "ins", &pvins, &pvt);
    f16_source(pvins[1], true);
  }
  std::vector<std::string> po, pot;
  op_group(*pv, "outs", &po, &pot);
  zero_fill(po[0], true);
  zero_fill(sum_init, true);
  zero_fill(qk_init, true);
  const Binding ob = output_storage(root.results[0]);
  const float scale = (float)(sq * sk);
  Dispatch d;
  d.ordinal = HXB_EXPORT_ATTENTION_F16;
  d.constants = {(uint32_t)BH, (uint32_t)Sq, (uint32_t)Skv, (uint32_t)D, 0u, f32_bits(scale)};
  d.bindings = {slice(qb, 0, (uint64_t)BH * Sq * D * 2), slice(kb, 0, (uint64_t)BH * Skv * D * 2),
                slice(vb, 0, (uint64_t)BH * Skv * D * 2), slice(ob, 0, (uint64_t)BH * Sq * D * 2)};
  out_->dispatches.push_back(std::move(d));
  std::ostringstream s;
  s << "attention_f16 dispatch: " << BH << " heads, " << Sq << " x " << Skv << " x " << D
    << ", scale " << sq << " * " << sk << " = " << scale << ", fully-masked rows -> 0 ("
    << chain.size() + 1 << " ops fused)";
  note("accept", root, s.str());
  return true;
}

bool FuncCompiler::has_bindings() const {
  for (const Op& op : f_.ops)
    if (op.name == "hal.interface.binding.subspan") return true;
  return false;
}

// A whole program (func.func over tensors, or an IREE entry over
// !hal.buffer_view): the arguments are the tensor arguments or the imported
// buffer views, the results the returned values (through hal.tensor.export
// and hal.tensor.barrier).
bool FuncCompiler::program_form(CompiledFunc* out) {
  std::vector<std::string> arg_vals;
  for (size_t a = 0; a < f_.arg_names.size(); ++a)
    if (parse_type(f_.arg_types[a]).tensor) arg_vals.push_back(f_.arg_names[a]);
  if (arg_vals.empty()) {
    std::vector<std::string> views;
    for (size_t a = 0; a < f_.arg_names.size(); ++a)
      if (f_.arg_types[a] == "!hal.buffer_view") views.push_back(f_.arg_names[a]);
    arg_vals.assign(views.size(), "");
    for (size_t i = 0; i < f_.ops.size(); ++i) {
      const Op& op = f_.ops[i];
      if (op.name != "hal.tensor.import" || op.results.empty()) continue;
      const auto o = op_operands(op);
      for (size_t v = 0; v < views.size(); ++v)
        if (!o.empty() && o.back() == views[v]) arg_vals[v] = op.results[0];
    }
  }
  for (size_t a = 0; a < arg_vals.size(); ++a) {
    const TensorType t = type_of(arg_vals[a]);
    if (!t.ok || !t.tensor || elem_code(t.elem) < 0) {
      log_ << "error @" << f_.name << ": argument " << a
           << " is not a static f16, f32 or i8 tensor\n";
      return false;
    }
    out->args.push_back(Desc{elem_code(t.elem), t.dims});
    storage_[arg_vals[a]] = Binding{kArg, (uint32_t)a, 0, type_bytes(t)};
  }
  // results: returned values (through hal.tensor.export / barrier)
  for (size_t i = 0; i < f_.ops.size(); ++i) {
    const Op& op = f_.ops[i];
    if (op.name != "return" && op.name != "func.return" && op.name != "util.return") continue;
    for (std::string v : op_operands(op)) {
      for (int guard = 0; guard < 4; ++guard) {
        const Op* d = def_op(v);
        if (!d) break;
        if (d->name == "hal.tensor.export") {
          v = op_operands(*d)[0];
        } else if (d->name == "hal.tensor.barrier") {
          std::vector<std::string> j, jt;
          op_group(*d, "join", &j, &jt);
          v = j.empty() ? v : j[0];
        } else {
          break;
        }
      }
      const TensorType t = type_of(v);
      if (!t.ok || !t.tensor || elem_code(t.elem) < 0) {
        err(op, "a returned value is not a static f16, f32 or i8 tensor");
        return false;
      }
      if (storage_.count(v)) {
        err(op, "returning an argument unchanged is not supported");
        return false;
      }
      storage_[v] = Binding{kResult, (uint32_t)out->results.size(), 0, type_bytes(t)};
      out->results.push_back(Desc{elem_code(t.elem), t.dims});
    }
  }
  return true;
}

// The dispatch form IREE hands a target backend's serializeExecutable: the
// operands are bindings declared by hal.interface.binding.subspan, read with
// *.dispatch.tensor.load and written with *.dispatch.tensor.store, whole
// (zero offsets, full sizes). Read-only bindings become the arguments and the
// others the results, each in binding order.
bool FuncCompiler::dispatch_form(CompiledFunc* out) {
  struct B {
    int binding;
    bool readonly;
    TensorType type;
    std::string value;  // the loaded or stored tensor
  };
  std::map<std::string, B> subspans;  // subspan result -> binding
  for (const Op& op : f_.ops) {
    if (op.name != "hal.interface.binding.subspan" || op.results.empty()) continue;
    int binding = -1;
    for (size_t i = 0; i + 2 < op.toks.size(); ++i)
      if (op.toks[i].k == Tok::kIdent && op.toks[i].s == "binding" && op.toks[i + 2].k == Tok::kNum)
        binding = atoi(op.toks[i + 2].s.c_str());
    const auto rt = op_result_types(op);
    // !iree_tensor_ext.dispatch.tensor<readonly:tensor<...>> (or flow's)
    const std::string t = rt.empty() ? "" : rt[0];
    const size_t colon = t.find(':'), open = t.find("tensor<", t.find('<') + 1);
    if (binding < 0 || colon == std::string::npos || open == std::string::npos) {
      err(op, "binding without an index or a dispatch tensor type");
      return false;
    }
    const std::string access = t.substr(t.find('<') + 1, colon - t.find('<') - 1);
    const TensorType tt = parse_type(t.substr(open, t.size() - open - 1));
    if (!tt.ok || elem_code(tt.elem) < 0) {
      err(op, "binding " + std::to_string(binding) + " is not a static f16, f32 or i8 tensor");
      return false;
    }
    subspans[op.results[0]] = B{binding, access == "readonly", tt, ""};
  }
  auto whole = [](const Op& op, const TensorType& t) {
    std::string sizes;
    for (const Tok& x : op_attr(op, "sizes")) sizes += x.s;
    std::string want = "[";
    for (size_t i = 0; i < t.dims.size(); ++i) want += (i ? "," : "") + std::to_string(t.dims[i]);
    want += "]";
    std::string offs;
    for (const Tok& x : op_attr(op, "offsets")) offs += x.s;
    for (char c : offs)
      if (c != '[' && c != ']' && c != ',' && c != '0') return false;
    return sizes == want;
  };
  for (const Op& op : f_.ops) {
    const bool load = op.name.size() > 20 && op.name.rfind(".dispatch.tensor.load") ==
                                                 op.name.size() - 21;
    const bool store = op.name.size() > 21 && op.name.rfind(".dispatch.tensor.store") ==
                                                  op.name.size() - 22;
    if (!load && !store) continue;
    const auto o = op_operands(op);
    const std::string target = load ? (o.empty() ? "" : o[0]) : (o.size() < 2 ? "" : o[1]);
    if (!subspans.count(target)) {
      err(op, "does not access a binding");
      return false;
    }
    B& b = subspans[target];
    if (!whole(op, b.type)) {
      err(op, "only whole-binding loads and stores are supported");
      return false;
    }
    b.value = load ? (op.results.empty() ? "" : op.results[0]) : o[0];
    consumed_.insert((int)(&op - &f_.ops[0]));
  }
  std::vector<B> in, res;
  for (auto& kv : subspans) (kv.second.readonly ? in : res).push_back(kv.second);
  auto by_binding = [](const B& x, const B& y) { return x.binding < y.binding; };
  std::sort(in.begin(), in.end(), by_binding);
  std::sort(res.begin(), res.end(), by_binding);
  for (const B& b : in) {
    storage_[b.value] = Binding{kArg, (uint32_t)out->args.size(), 0, type_bytes(b.type)};
    out->args.push_back(Desc{elem_code(b.type.elem), b.type.dims});
    log_ << "binding " << b.binding << " -> argument " << out->args.size() - 1 << "\n";
  }
  for (const B& b : res) {
    if (b.value.empty()) continue;
    storage_[b.value] = Binding{kResult, (uint32_t)out->results.size(), 0, type_bytes(b.type)};
    out->results.push_back(Desc{elem_code(b.type.elem), b.type.dims});
    log_ << "binding " << b.binding << " -> result " << out->results.size() - 1 << "\n";
  }
  return true;
}

bool FuncCompiler::run(CompiledFunc* out) {
  out_ = out;
  out->name = f_.name;
  // definitions, types and uses
  for (size_t a = 0; a < f_.arg_names.size(); ++a) {
    defs_[f_.arg_names[a]] = Def{-1, (int)a};
    types_[f_.arg_names[a]] = f_.arg_types[a];
  }
  for (size_t i = 0; i < f_.ops.size(); ++i) {
    const Op& op = f_.ops[i];
    auto rt = op_result_types(op);
    std::vector<std::string> outs, outs_t;
    if (rt.empty() && op_group(op, "outs", &outs, &outs_t)) rt = outs_t;  // linalg.transpose
    if (op.name == "hal.tensor.barrier") {
      std::vector<std::string> j, jt;
      op_group(op, "join", &j, &jt);
      rt = jt;
    }
    for (size_t r = 0; r < op.results.size(); ++r) {
      defs_[op.results[r]] = Def{(int)i, -1};
      if (r < rt.size()) types_[op.results[r]] = rt[r];
    }
    std::vector<std::string> names, ts;
    for (const char* kw : {"ins", "outs", "join"})
      if (op_group(op, kw, &names, &ts))
        for (const auto& n : names) uses_[n]++;
    for (const auto& n : op_operands(op)) uses_[n]++;
  }
  // The dispatch form IREE hands a target backend: bindings declared by
  // hal.interface.binding.subspan, read with dispatch.tensor.load and written
  // with dispatch.tensor.store. Read-only bindings become the arguments and
  // the others the results, each in binding order.
  // The dispatch form IREE hands a target backend, or a whole program
  if (has_bindings()) {
    if (!dispatch_form(out)) return false;
  } else if (!program_form(out)) {
    return false;
  }
  // dispatch formation, in program order: attention chains first (their
  // inner batch_matmuls are not standalone matmuls), then int8-weight and
  // f16 contractions
  bool ok = true;
  for (size_t i = 0; i < f_.ops.size() && ok; ++i)
    if (!consumed_.count((int)i) && f_.ops[i].name == "linalg.generic") try_attention((int)i);
  for (size_t i = 0; i < f_.ops.size() && ok; ++i) {
    if (consumed_.count((int)i)) continue;
    const std::string& n = f_.ops[i].name;
    if (n == "linalg.generic" && try_w8((int)i)) continue;
    if (n.rfind("linalg.", 0) == 0 && n != "linalg.fill" && n != "linalg.index" &&
        n != "linalg.yield") {
      const size_t before = out->dispatches.size();
      try_contraction((int)i);
      if (out->dispatches.size() == before && !consumed_.count((int)i)) {
        // not a dispatch the target forms
      }
    }
  }
  // everything else must be glue the dispatches made redundant
  static const std::set<std::string> glue = {
      "arith.constant", "tensor.empty", "hal.tensor.import", "hal.tensor.export",
      "hal.tensor.barrier", "return", "func.return", "util.return",
      "hal.interface.binding.subspan"};
  for (size_t i = 0; i < f_.ops.size(); ++i) {
    if (consumed_.count((int)i) || glue.count(f_.ops[i].name)) continue;
    const Op& op = f_.ops[i];
    // a fill or elementwise op whose every user was fused away
    bool dead = !op.results.empty();
    for (const auto& r : op.results) {
      for (size_t j = 0; j < f_.ops.size(); ++j) {
        if (consumed_.count((int)j) || j == i) continue;
        std::vector<std::string> names, ts;
        bool used = false;
        for (const char* kw : {"ins", "outs", "join"})
          if (op_group(f_.ops[j], kw, &names, &ts))
            for (const auto& n : names) used |= n == r;
        for (const auto& n : op_operands(f_.ops[j])) used |= n == r;
        if (used) dead = false;
      }
    }
    if (dead && (op.name == "linalg.fill" || op.name == "tensor.expand_shape")) continue;
    err(op, "no B200 dispatch for this operation");
    ok = false;
  }
  if (ok && out->dispatches.empty()) {
    log_ << "error @" << f_.name << ": no dispatch formed\n";
    ok = false;
  }
  return ok;
}

// ----------------------------------------------------------- serialisation
void put32(std::vector<uint8_t>* b, uint32_t v) {
  for (int i = 0; i < 4; ++i) b->push_back((uint8_t)(v >> (8 * i)));
}
void put64(std::vector<uint8_t>* b, uint64_t v) {
  for (int i = 0; i < 8; ++i) b->push_back((uint8_t)(v >> (8 * i)));
}
void put_str(std::vector<uint8_t>* b, const std::string& s) {
  put32(b, (uint32_t)s.size());
  b->insert(b->end(), s.begin(), s.end());
}

std::vector<uint8_t> serialise(const std::vector<CompiledFunc>& funcs) {
  std::vector<uint8_t> b(kMagic, kMagic + 4);
  put32(&b, kBlobVersion);
  put_str(&b, HXB_EXECUTABLE_FORMAT);
  put32(&b, (uint32_t)funcs.size());
  for (const CompiledFunc& f : funcs) {
    put_str(&b, f.name);
    for (const auto* list : {&f.args, &f.results}) {
      put32(&b, (uint32_t)list->size());
      for (const Desc& d : *list) {
        put32(&b, (uint32_t)d.elem);
        put32(&b, (uint32_t)d.dims.size());
        for (long long x : d.dims) put64(&b, (uint64_t)x);
      }
    }
    put32(&b, (uint32_t)f.transients.size());
    for (uint64_t t : f.transients) put64(&b, t);
    put32(&b, (uint32_t)f.dispatches.size());
    for (const Dispatch& d : f.dispatches) {
      put32(&b, d.ordinal);
      put32(&b, (uint32_t)d.constants.size());
      for (uint32_t c : d.constants) put32(&b, c);
      put32(&b, (uint32_t)d.bindings.size());
      for (const Binding& x : d.bindings) {
        put32(&b, x.kind);
        put32(&b, x.index);
        put64(&b, x.offset);
        put64(&b, x.length);
      }
    }
  }
  return b;
}

char* dup_string(const std::string& s) {
  char* p = static_cast<char*>(malloc(s.size() + 1));
  if (p) memcpy(p, s.c_str(), s.size() + 1);
  return p;
}

}  // namespace
}  // namespace hxbc

extern "C" void hxb_compiler_options_initialize(hxb_compiler_options_t* o) {
  if (!o) return;
  o->enable_matmul = 1;
  o->enable_w8a16 = 1;
  o->enable_attention = 1;
  o->num_sms = 0;
}

extern "C" hxb_status_t hxb_compile_mlir(const char* text, size_t length,
                                         const hxb_compiler_options_t* options,
                                         void** out_executable, size_t* out_size,
                                         char** out_log) {
  using namespace hxbc;
  if (out_executable) *out_executable = nullptr;
  if (out_size) *out_size = 0;
  if (out_log) *out_log = nullptr;
  if (!text || !out_executable || !out_size) return HXB_STATUS_INVALID_ARGUMENT;
  hxb_compiler_options_t opt;
  hxb_compiler_options_initialize(&opt);
  if (options) opt = *options;
  std::ostringstream log;
  Module m;
  std::string perr;
  hxb_status_t status = HXB_OK;
  std::vector<CompiledFunc> funcs;
  if (!parse_module(std::string(text, length), &m, &perr)) {
    log << "error: " << perr << "\n";
    status = HXB_STATUS_INVALID_ARGUMENT;
  } else {
    for (const Func& f : m.funcs) {
      FuncCompiler fc(m, f, opt, log);
      if (!fc.has_linalg()) {
        log << "skip @" << f.name << " line " << f.line << ": no linalg ops (a wrapper)\n";
        continue;
      }
      CompiledFunc cf;
      if (!fc.run(&cf)) {
        status = HXB_STATUS_UNSUPPORTED;
        continue;
      }
      log << "function @" << f.name << ": " << cf.dispatches.size() << " dispatch(es), "
          << cf.args.size() << " argument(s), " << cf.results.size() << " result(s), "
          << cf.transients.size() << " transient buffer(s)\n";
      funcs.push_back(std::move(cf));
    }
    if (status == HXB_OK && funcs.empty()) {
      log << "error: no function with dispatches\n";
      status = HXB_STATUS_UNSUPPORTED;
    }
  }
  if (status == HXB_OK) {
    const std::vector<uint8_t> blob = serialise(funcs);
    void* p = malloc(blob.size());
    if (!p) {
      status = HXB_STATUS_RESOURCE_EXHAUSTED;
    } else {
      memcpy(p, blob.data(), blob.size());
      *out_executable = p;
      *out_size = blob.size();
    }
  }
  if (out_log) *out_log = dup_string(log.str());
  return status;
}

extern "C" void hxb_compiler_free(void* p) { free(p); }

extern "C" hxb_status_t hxb_executable_binary_mlir(const void* executable, size_t size,
                                                   const char* symbol, char** out_text) {
  if (!executable || size < 8 || !out_text) return HXB_STATUS_INVALID_ARGUMENT;
  if (memcmp(executable, hxbc::kMagic, 4) != 0) return HXB_STATUS_INVALID_ARGUMENT;
  std::ostringstream s;
  s << "hal.executable.binary @" << (symbol && *symbol ? symbol : "b200") << " attributes {data = dense<[";
  const int8_t* b = static_cast<const int8_t*>(executable);
  for (size_t i = 0; i < size; ++i) s << (i ? ", " : "") << (int)b[i];
  s << "]> : vector<" << size << "xi8>, format = \"" << HXB_EXECUTABLE_FORMAT
    << "\", mime_type = \"" << HXB_EXECUTABLE_MIME_TYPE << "\"}\n";
  *out_text = hxbc::dup_string(s.str());
  return *out_text ? HXB_OK : HXB_STATUS_RESOURCE_EXHAUSTED;
}

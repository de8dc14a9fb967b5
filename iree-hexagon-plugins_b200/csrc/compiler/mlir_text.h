// A reader for the textual MLIR the B200 target compiles: the pretty-printed
// form of builtin.module, func.func / util.func, and the linalg, arith,
// math, tensor and hal.tensor ops of linalg-on-tensors programs (the inputs
// of the reference's compiler, e.g. examples/matmul/matmul.mlir and
// examples/attention_layer/attention_layer.mlir).
//
// It does not implement MLIR's grammar. It tokenises the text, splits every
// block into operations (an operation starts a line with its results or its
// dotted name and runs, across lines, until the next such line at bracket
// depth 0), keeps each operation's tokens, and parses the single-block
// regions of linalg.generic. The pattern matcher (recognize.cc) reads
// operands, types and attributes from those tokens.
#pragma once

#include <map>
#include <string>
#include <vector>

namespace hxbc {

struct Tok {
  enum Kind { kIdent, kSsa, kSym, kHash, kStr, kNum, kPunct, kAngle, kCaret, kBang, kEnd };
  Kind k;
  std::string s;
  int line;
  bool bol;  // first token of its line
};

struct Op;

struct Block {
  std::vector<std::string> args;       // %in, %out, ...
  std::vector<std::string> arg_types;  // f16, f32, ...
  std::vector<Op> ops;
};

struct Op {
  std::vector<std::string> results;  // "%4", or "%17#0", "%17#1" for %17:2
  std::string name;                  // "linalg.generic", "return", ...
  int line = 0;
  std::vector<Tok> toks;             // tokens after the name, regions removed
  std::vector<Block> region;         // the op's region (one block), if any
};

struct Func {
  std::string name;  // without '@'
  int line = 0;
  std::vector<std::string> arg_names, arg_types, result_types;
  std::vector<Op> ops;
};

struct Module {
  std::map<std::string, std::string> aliases;  // "#map1" -> "affine_map<...>"
  std::vector<Func> funcs;
};

// Parses `text`; on failure returns false with `error` set ("line N: ...").
bool parse_module(const std::string& text, Module* out, std::string* error);

// ------------------------------------------------------------ op queries
// Operand names and types of a `kw(%a, %b : t1, t2)` group (kw = "ins",
// "outs", "join", "wait"); false if the op has no such group.
bool op_group(const Op& op, const std::string& kw, std::vector<std::string>* names,
              std::vector<std::string>* types);
// Plain SSA operands of the op (in order, outside any keyword group and
// outside the attribute dictionary), e.g. the operands of arith.mulf.
std::vector<std::string> op_operands(const Op& op);
// Result types: the type(s) after the last depth-0 "->", else the last
// depth-0 type after ':' (arith ops, constants, tensor.empty).
std::vector<std::string> op_result_types(const Op& op);
// Raw token text of attribute `key` in the op's attribute dictionary
// ({key = value, ...}) or of a trailing `key = value` (permutation), or "".
std::vector<Tok> op_attr(const Op& op, const std::string& key);
// The value token of arith.constant (number, hex, true/false, dense<...>).
std::string op_constant_text(const Op& op);

// ------------------------------------------------------------ types
struct TensorType {
  bool ok = false;
  bool tensor = false;  // false: scalar
  std::vector<long long> dims;
  std::string elem;     // "f16", "f32", "f64", "i8", "i1", "i64", "index"
};
TensorType parse_type(const std::string& t);

// An affine map (d0, ..., dn-1) -> (e0, ...): each result a dim index or -1
// for the constant 0.
struct AffineMap {
  bool ok = false;
  int num_dims = 0;
  std::vector<int> results;
};
AffineMap parse_affine_map(const std::string& text);

}  // namespace hxbc

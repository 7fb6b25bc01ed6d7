// StableHLO text front door: sb_module_load_stablehlo.
//
// Replaces `iree-compile` + `load_vmfb` (sheaf/src/runtime/jit/vag.rs:660-726,
// sheaf/src/runtime/iree_session.rs:307-340) for the text Sheaf's emitter
// prints (sheaf/src/lowering/stablehlo/emit.rs:240-257 and the op printers in
// that directory). Three parts:
//   1. A parser for the op surface of that emitter (elementwise, convert,
//      clamp, broadcast_in_dim, reshape, transpose, reverse, iota,
//      concatenate, slice, pad, dynamic_slice, dynamic_update_slice,
//      dot_general, reduce, compare, select, constant, generic gather, the
//      two-result sort of top_k, return), multi-line generic ops included.
//   2. A generic executor: each op runs as a library kernel in its declared
//      element type (so bf16 modules round after every op, as the reference
//      executes them); intermediates live in one device arena planned by
//      liveness, reshapes alias their operand, dot_general is canonicalised
//      to [batch, M, K] x [batch, K, N] and runs on the tcgen05 / FFMA GEMM
//      when unbatched (a generic batched kernel otherwise).
//   3. A recognizer: a `value_and_grad` function whose signature is the
//      nanoGPT pytree (params leaves, then x / y token ids; outputs loss then
//      one gradient per leaf, jit/vag.rs:126-141,565-574) is mapped onto the
//      fused nanoGPT plan (gpt_vag.cpp). The first call runs both the fused
//      plan and the generic executor on the same inputs and keeps the fused
//      plan only if every output agrees; otherwise the module stays generic.
// An op outside the surface returns UNIMPLEMENTED, which the caller treats as
// a failed compile (jit/compile.rs:119-125).
//
// Plan cache: with SHEAF_B200_CACHE_DIR set, the outcome of the first-call
// check is recorded in <dir>/manifest.json, keyed by a hash of the module
// text, the function name and the bytes of this library (the counterpart of
// the reference's __sheaf__/manifest.json of compiled modules,
// jit/compile.rs:419-478). A later load of the same text by the same build
// starts from the recorded plan: a verified fused plan runs from the first
// call, a rejected one is not built.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <dlfcn.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <functional>
#include <map>
#include <mutex>
#include <memory>
#include <sstream>
#include <string>
#include <vector>

#include "hlo_kernels.h"
#include "runtime.h"
#include "sb_kernels.h"
#include "sb_nn.h"

namespace sb {

namespace {

using namespace hlo;

// ---------------------------------------------------------------------------
// IR
// ---------------------------------------------------------------------------

struct TType {
  int dt = DT_F32;
  std::vector<int64_t> shape;
  int64_t numel() const {
    int64_t n = 1;
    for (auto d : shape) n *= d;
    return n;
  }
  size_t bytes() const { return static_cast<size_t>(numel()) * dt_size(dt); }
  bool operator==(const TType& o) const { return dt == o.dt && shape == o.shape; }
};

uint32_t elem_of(int dt) {
  switch (dt) {
    case DT_F32: return SB_ELEM_F32;
    case DT_BF16: return SB_ELEM_BF16;
    case DT_F16: return SB_ELEM_F16;
    case DT_I32: return SB_ELEM_I32;
    default: return 0;
  }
}

struct HOp {
  std::string kind;
  std::string result;
  std::string result2;  // second result (sort's permuted payload)
  TType type2;
  bool descending = true;  // sort: GT comparator
  std::vector<std::string> operands;
  TType type;
  std::vector<TType> operand_types;
  std::vector<int64_t> dims;
  std::vector<int64_t> lb, rb, lc, rc;
  std::vector<int64_t> starts, limits, strides;
  std::vector<int64_t> low, high, interior;
  int64_t dim = 0;
  int cmp = C_EQ;
  int reduce_op = B_ADD;
  int unary_op = U_COPY;
  int binary_op = B_ADD;
  std::vector<double> values;
  std::vector<int64_t> offset_dims, slice_sizes, collapsed, start_index_map, operand_batching;
  int64_t index_vector_dim = -1;
  std::string text;
};

struct HFunc {
  std::string name;
  std::vector<std::string> arg_names;
  std::vector<TType> args;
  std::vector<TType> rets;
  std::vector<HOp> ops;
  std::vector<std::string> ret_names;
};

struct HModule {
  std::string name;
  std::vector<HFunc> funcs;
};

struct ParseError {
  std::string msg;
};

// ---------------------------------------------------------------------------
// Parser
// ---------------------------------------------------------------------------

class Cursor {
 public:
  explicit Cursor(const std::string& s) : s_(s) {}
  void ws() {
    while (p_ < s_.size() && std::isspace(static_cast<unsigned char>(s_[p_]))) ++p_;
  }
  bool eof() {
    ws();
    return p_ >= s_.size();
  }
  bool peek(const char* t) {
    ws();
    return s_.compare(p_, std::strlen(t), t) == 0;
  }
  bool accept(const char* t) {
    if (!peek(t)) return false;
    p_ += std::strlen(t);
    return true;
  }
  void expect(const char* t) {
    if (!accept(t)) fail(std::string("expected '") + t + "'");
  }
  [[noreturn]] void fail(const std::string& m) {
    throw ParseError{m + " at: " + s_.substr(p_, 60)};
  }
  std::string ident() {
    ws();
    size_t b = p_;
    while (p_ < s_.size() && (std::isalnum(static_cast<unsigned char>(s_[p_])) || s_[p_] == '_' || s_[p_] == '.' ||
                              s_[p_] == '$' || s_[p_] == '-'))
      ++p_;
    if (b == p_) fail("expected identifier");
    return s_.substr(b, p_ - b);
  }
  std::string value() {  // %name
    ws();
    if (p_ >= s_.size() || s_[p_] != '%') fail("expected %value");
    size_t b = p_++;
    while (p_ < s_.size() && (std::isalnum(static_cast<unsigned char>(s_[p_])) || s_[p_] == '_' || s_[p_] == '#'))
      ++p_;
    return s_.substr(b, p_ - b);
  }
  int64_t integer() {
    ws();
    size_t b = p_;
    if (p_ < s_.size() && (s_[p_] == '-' || s_[p_] == '+')) ++p_;
    while (p_ < s_.size() && std::isdigit(static_cast<unsigned char>(s_[p_]))) ++p_;
    if (b == p_) fail("expected integer");
    return std::stoll(s_.substr(b, p_ - b));
  }
  std::vector<int64_t> int_list() {  // [a, b, ...]
    std::vector<int64_t> v;
    expect("[");
    if (accept("]")) return v;
    do v.push_back(integer());
    while (accept(","));
    expect("]");
    return v;
  }
  TType type() {
    expect("tensor<");
    TType t;
    std::string body;
    ws();
    while (p_ < s_.size() && s_[p_] != '>') body += s_[p_++];
    expect(">");
    // body = "2x3xf32" | "f32"
    size_t last = body.rfind('x');
    std::string et = body;
    if (last != std::string::npos) {
      // split on 'x' but element types contain no 'x'
      std::vector<std::string> parts;
      size_t b = 0;
      for (size_t i = 0; i <= body.size(); ++i)
        if (i == body.size() || body[i] == 'x') {
          parts.push_back(body.substr(b, i - b));
          b = i + 1;
        }
      et = parts.back();
      for (size_t i = 0; i + 1 < parts.size(); ++i) {
        if (parts[i].empty() || !std::isdigit(static_cast<unsigned char>(parts[i][0])))
          fail("dynamic or malformed dimension in tensor type");
        t.shape.push_back(std::stoll(parts[i]));
      }
    }
    if (et == "f32") t.dt = DT_F32;
    else if (et == "bf16") t.dt = DT_BF16;
    else if (et == "f16") t.dt = DT_F16;
    else if (et == "i32" || et == "ui32") t.dt = DT_I32;
    else if (et == "i1") t.dt = DT_I1;
    else fail("unsupported element type " + et);
    return t;
  }
  std::vector<TType> type_list() {  // (T, U) or T
    std::vector<TType> v;
    if (accept("(")) {
      if (accept(")")) return v;
      do v.push_back(type());
      while (accept(","));
      expect(")");
    } else {
      v.push_back(type());
    }
    return v;
  }
  size_t pos() const { return p_; }
  const std::string& str() const { return s_; }
  void set(size_t p) { p_ = p; }

 private:
  const std::string& s_;
  size_t p_ = 0;
};

std::string strip_comments(const char* text, size_t len) {
  std::string out;
  out.reserve(len);
  for (size_t i = 0; i < len; ++i) {
    if (text[i] == '/' && i + 1 < len && text[i + 1] == '/') {
      while (i < len && text[i] != '\n') ++i;
      out += '\n';
      continue;
    }
    out += text[i];
  }
  return out;
}

const std::map<std::string, int>& unary_ops() {
  static const std::map<std::string, int> m = {
      {"negate", U_NEG}, {"abs", U_ABS}, {"exponential", U_EXP}, {"log", U_LOG}, {"sqrt", U_SQRT},
      {"rsqrt", U_RSQRT}, {"tanh", U_TANH}, {"sine", U_SIN}, {"cosine", U_COS}, {"floor", U_FLOOR},
      {"ceil", U_CEIL}, {"sign", U_SIGN}, {"logistic", U_LOGISTIC}, {"not", U_NOT}, {"log_plus_one", U_LOG1P},
      {"exponential_minus_one", U_EXPM1}};
  return m;
}

const std::map<std::string, int>& binary_ops() {
  static const std::map<std::string, int> m = {
      {"add", B_ADD},      {"subtract", B_SUB},   {"multiply", B_MUL},        {"divide", B_DIV},
      {"power", B_POW},    {"maximum", B_MAX},    {"minimum", B_MIN},         {"remainder", B_REM},
      {"floor_divide", B_FLOORDIV}, {"atan2", B_ATAN2}, {"and", B_AND},       {"or", B_OR},
      {"xor", B_XOR},      {"shift_left", B_SHL}, {"shift_right_logical", B_SHR}};
  return m;
}

void parse_dense(Cursor& c, HOp& op) {
  // dense<v> | dense<0x...> | dense<[[...]]> | dense<true>
  c.expect("dense<");
  const std::string& s = c.str();
  size_t p = c.pos();
  int depth = 0;
  std::string body;
  while (p < s.size()) {
    if (s[p] == '<') depth++;
    if (s[p] == '>') {
      if (depth == 0) break;
      depth--;
    }
    body += s[p++];
  }
  c.set(p);
  c.expect(">");
  std::string tok;
  auto flush = [&]() {
    if (tok.empty()) return;
    if (tok == "true") op.values.push_back(1.0);
    else if (tok == "false") op.values.push_back(0.0);
    else if (tok.size() > 2 && tok[0] == '0' && (tok[1] == 'x' || tok[1] == 'X')) {
      const uint64_t bits = std::stoull(tok.substr(2), nullptr, 16);
      op.values.push_back(std::nan(""));  // placeholder; raw bits kept below
      op.dims.push_back(static_cast<int64_t>(bits));  // raw bit pattern(s)
      op.dim = 1;                                      // marks hex constants
    } else {
      op.values.push_back(std::stod(tok));
    }
    tok.clear();
  };
  for (char ch : body) {
    if (ch == '[' || ch == ']' || ch == ',' || std::isspace(static_cast<unsigned char>(ch))) {
      flush();
    } else {
      tok += ch;
    }
  }
  flush();
}

HOp parse_op(const std::string& stmt) {
  Cursor c(stmt);
  HOp op;
  op.text = stmt.size() > 160 ? stmt.substr(0, 160) : stmt;
  op.result = c.value();
  if (c.accept(",")) op.result2 = c.value();
  c.expect("=");
  // operands of a quoted op: ( %a, %b, ... )
  auto paren_values = [&]() {
    c.expect("(");
    if (!c.accept(")")) {
      do op.operands.push_back(c.value());
      while (c.accept(","));
      c.expect(")");
    }
  };
  if (c.accept("\"stablehlo.dynamic_slice\"")) {
    // "stablehlo.dynamic_slice"(%x, %i0, ...) { slice_sizes = array<i64: ...> } : (...) -> R
    // (indexing_ops.rs:289-318)
    op.kind = "dynamic_slice";
    paren_values();
    c.expect("{");
    c.expect("slice_sizes");
    c.expect("=");
    c.expect("array<i64:");
    do op.slice_sizes.push_back(c.integer());
    while (c.accept(","));
    c.expect(">");
    c.expect("}");
    c.expect(":");
    op.operand_types = c.type_list();
    c.expect("->");
    op.type = c.type();
    return op;
  }
  if (c.accept("\"stablehlo.dynamic_update_slice\"")) {
    // "stablehlo.dynamic_update_slice"(%x, %u, %i0, ...) : (...) -> T (indexing_ops.rs:320-343)
    op.kind = "dynamic_update_slice";
    paren_values();
    c.expect(":");
    op.operand_types = c.type_list();
    c.expect("->");
    op.type = c.type();
    return op;
  }
  if (c.accept("\"stablehlo.sort\"")) {
    // %v, %i = "stablehlo.sort"(%keys, %payload) ({ ^bb0(...): %p = "stablehlo.compare"(%a, %b)
    //   {comparison_direction = #stablehlo<comparison_direction GT>} ... "stablehlo.return"(%p) ... })
    //   {dimension = d : i64, is_stable = true} : (T, I) -> (T, I)   (indexing_ops.rs:486-550)
    op.kind = "sort";
    paren_values();
    c.expect("(");
    // the comparator region: the block's first two arguments are the key
    // pair; only a GT or LT compare of that pair is accepted
    const std::string& s = c.str();
    size_t p = c.pos();
    int depth = 1;
    const size_t body0 = p;
    while (p < s.size() && depth > 0) {
      if (s[p] == '(' || s[p] == '{') depth++;
      if (s[p] == ')' || s[p] == '}') depth--;
      ++p;
    }
    const std::string body = s.substr(body0, p - body0);
    c.set(p);
    Cursor rc(body);
    rc.expect("{");
    rc.expect("^bb0(");
    std::vector<std::string> args;
    do {
      args.push_back(rc.value());
      rc.expect(":");
      rc.type();
    } while (rc.accept(","));
    rc.expect(")");
    rc.expect(":");
    const std::string pred = rc.value();
    rc.expect("=");
    rc.expect("\"stablehlo.compare\"(");
    const std::string lhs = rc.value();
    rc.expect(",");
    const std::string rhs = rc.value();
    rc.expect(")");
    rc.expect("{");
    rc.expect("comparison_direction");
    rc.expect("=");
    rc.expect("#stablehlo<comparison_direction");
    const std::string dir = rc.ident();
    if (args.size() != 4 || lhs != args[0] || rhs != args[1] || (dir != "GT" && dir != "LT"))
      c.fail("sort comparator must be a GT or LT compare of the key pair");
    op.descending = dir == "GT";
    (void)pred;
    c.expect("{");
    while (!c.accept("}")) {
      const std::string k = c.ident();
      c.expect("=");
      if (k == "dimension") {
        op.dim = c.integer();
        if (c.accept(":")) c.ident();
      } else if (k == "is_stable") {
        c.ident();
      } else {
        c.fail("unknown sort attribute " + k);
      }
      c.accept(",");
    }
    c.expect(":");
    op.operand_types = c.type_list();
    c.expect("->");
    const auto rt = c.type_list();
    if (rt.size() != 2 || op.result2.empty()) c.fail("sort must return (keys, payload)");
    op.type = rt[0];
    op.type2 = rt[1];
    return op;
  }
  if (!op.result2.empty()) c.fail("only stablehlo.sort has two results");
  if (c.accept("\"stablehlo.gather\"")) {
    op.kind = "gather";
    c.expect("(");
    op.operands.push_back(c.value());
    c.expect(",");
    op.operands.push_back(c.value());
    c.expect(")");
    c.expect("{");
    // attribute dictionary
    while (!c.accept("}")) {
      std::string key = c.ident();
      c.expect("=");
      if (key == "dimension_numbers") {
        c.expect("#stablehlo.gather<");
        while (!c.accept(">")) {
          std::string k = c.ident();
          c.expect("=");
          if (k == "index_vector_dim") {
            op.index_vector_dim = c.integer();
          } else {
            auto v = c.int_list();
            if (k == "offset_dims") op.offset_dims = v;
            else if (k == "collapsed_slice_dims") op.collapsed = v;
            else if (k == "start_index_map") op.start_index_map = v;
            else if (k == "operand_batching_dims") op.operand_batching = v;
            else if (k == "start_indices_batching_dims") {
              if (!v.empty()) c.fail("batched gather is not supported");
            }
          }
          c.accept(",");
        }
      } else if (key == "slice_sizes") {
        c.expect("array<i64:");
        do op.slice_sizes.push_back(c.integer());
        while (c.accept(","));
        c.expect(">");
      } else if (key == "indices_are_sorted") {
        c.ident();
      } else {
        c.fail("unknown gather attribute " + key);
      }
      c.accept(",");
    }
    c.expect(":");
    op.operand_types = c.type_list();
    c.expect("->");
    op.type = c.type();
    return op;
  }
  c.expect("stablehlo.");
  std::string name;
  {
    // op names are lowercase words joined by '_'
    c.ws();
    const std::string& s = c.str();
    size_t p = c.pos();
    while (p < s.size() && (std::isalnum(static_cast<unsigned char>(s[p])) || s[p] == '_')) name += s[p++];
    c.set(p);
  }
  op.kind = name;
  // ": (T, U) -> V" | ": T" | ": I1, T" (select); the result type is V or the
  // last listed type.
  auto ends_with_types = [&](bool arrow) {
    c.expect(":");
    op.operand_types = c.type_list();
    while (c.accept(",")) op.operand_types.push_back(c.type());
    if (arrow && c.accept("->"))
      op.type = c.type();
    else
      op.type = op.operand_types.back();
  };
  if (unary_ops().count(name)) {
    op.kind = "unary";
    op.unary_op = unary_ops().at(name);
    op.operands.push_back(c.value());
    ends_with_types(true);
  } else if (binary_ops().count(name)) {
    op.kind = "binary";
    op.binary_op = binary_ops().at(name);
    op.operands.push_back(c.value());
    c.expect(",");
    op.operands.push_back(c.value());
    ends_with_types(true);
  } else if (name == "convert" || name == "reshape") {
    op.operands.push_back(c.value());
    ends_with_types(true);
  } else if (name == "clamp") {
    for (int i = 0; i < 3; ++i) {
      op.operands.push_back(c.value());
      if (i < 2) c.expect(",");
    }
    ends_with_types(true);
  } else if (name == "broadcast_in_dim" || name == "transpose") {
    op.operands.push_back(c.value());
    c.expect(",");
    c.expect("dims");
    c.expect("=");
    op.dims = c.int_list();
    ends_with_types(true);
  } else if (name == "reverse") {
    // stablehlo.reverse %a, dims = [d] : (T) -> T (indexing_ops.rs:184-205)
    op.operands.push_back(c.value());
    c.expect(",");
    c.expect("dims");
    c.expect("=");
    op.dims = c.int_list();
    ends_with_types(true);
  } else if (name == "dynamic_update_slice") {
    // stablehlo.dynamic_update_slice %x, %u, %i0, ... : (T, U, tensor<i32>, ...) -> T
    // (indexing_ops.rs:207-287)
    do op.operands.push_back(c.value());
    while (c.accept(","));
    ends_with_types(true);
  } else if (name == "iota") {
    c.expect("dim");
    c.expect("=");
    op.dim = c.integer();
    c.expect(":");
    op.type = c.type();
  } else if (name == "concatenate") {
    do {
      op.operands.push_back(c.value());
      c.expect(",");
    } while (c.peek("%"));
    c.expect("dim");
    c.expect("=");
    op.dim = c.integer();
    ends_with_types(true);
  } else if (name == "slice") {
    op.operands.push_back(c.value());
    c.expect("[");
    do {
      op.starts.push_back(c.integer());
      c.expect(":");
      op.limits.push_back(c.integer());
      if (c.accept(":")) op.strides.push_back(c.integer());
      else op.strides.push_back(1);
    } while (c.accept(","));
    c.expect("]");
    ends_with_types(true);
  } else if (name == "pad") {
    op.operands.push_back(c.value());
    c.expect(",");
    op.operands.push_back(c.value());
    while (c.accept(",")) {
      std::string k = c.ident();
      c.expect("=");
      auto v = c.int_list();
      if (k == "low") op.low = v;
      else if (k == "high") op.high = v;
      else if (k == "interior") op.interior = v;
    }
    ends_with_types(true);
  } else if (name == "dot_general") {
    op.operands.push_back(c.value());
    c.expect(",");
    op.operands.push_back(c.value());
    while (c.accept(",")) {
      std::string k = c.ident();
      c.expect("=");
      if (k == "batching_dims" || k == "contracting_dims") {
        auto a = c.int_list();
        c.expect("x");
        auto b = c.int_list();
        if (k == "batching_dims") {
          op.lb = a;
          op.rb = b;
        } else {
          op.lc = a;
          op.rc = b;
        }
      } else {
        // precision / algorithm attributes: skip to the next ',' or ':'
        int depth = 0;
        const std::string& s = c.str();
        size_t p = c.pos();
        while (p < s.size() && !(depth == 0 && (s[p] == ',' || s[p] == ':'))) {
          if (s[p] == '[' || s[p] == '<' || s[p] == '(') depth++;
          if (s[p] == ']' || s[p] == '>' || s[p] == ')') depth--;
          ++p;
        }
        c.set(p);
      }
    }
    ends_with_types(true);
  } else if (name == "reduce") {
    c.expect("(");
    op.operands.push_back(c.value());
    c.expect("init:");
    op.operands.push_back(c.value());
    c.expect(")");
    c.expect("applies");
    c.expect("stablehlo.");
    const std::string r = c.ident();
    if (r == "add") op.reduce_op = B_ADD;
    else if (r == "maximum") op.reduce_op = B_MAX;
    else if (r == "minimum") op.reduce_op = B_MIN;
    else if (r == "multiply") op.reduce_op = B_MUL;
    else if (r == "and") op.reduce_op = B_AND;
    else if (r == "or") op.reduce_op = B_OR;
    else c.fail("unsupported reduction " + r);
    c.expect("across");
    c.expect("dimensions");
    c.expect("=");
    op.dims = c.int_list();
    ends_with_types(true);
  } else if (name == "compare") {
    const std::string dir = c.ident();
    static const std::map<std::string, int> dirs = {{"EQ", C_EQ}, {"NE", C_NE}, {"LT", C_LT},
                                                    {"LE", C_LE}, {"GT", C_GT}, {"GE", C_GE}};
    if (!dirs.count(dir)) c.fail("comparison direction");
    op.cmp = dirs.at(dir);
    c.expect(",");
    op.operands.push_back(c.value());
    c.expect(",");
    op.operands.push_back(c.value());
    if (c.accept(",")) c.ident();  // comparison type
    ends_with_types(true);
  } else if (name == "select") {
    for (int i = 0; i < 3; ++i) {
      op.operands.push_back(c.value());
      if (i < 2) c.expect(",");
    }
    ends_with_types(true);
  } else if (name == "constant") {
    parse_dense(c, op);
    c.expect(":");
    op.type = c.type();
  } else {
    c.fail("op stablehlo." + name + " is not supported by the sm_100a library");
  }
  return op;
}

HModule parse_module(const char* text, size_t len) {
  const std::string src = strip_comments(text, len);
  HModule m;
  Cursor c(src);
  // a bare func.func (as printed in the reference's docs) is an implicit module
  const bool bare = c.peek("func.func");
  if (!bare) {
    c.expect("module");
    if (c.peek("@")) {
      c.expect("@");
      m.name = c.ident();
    }
    // optional attributes before '{'
    while (!c.accept("{")) {
      if (c.eof()) c.fail("expected '{'");
      c.set(c.pos() + 1);
    }
  }
  while (true) {
    if (bare ? c.eof() : c.accept("}")) break;
    if (c.eof()) c.fail("unterminated module");
    c.expect("func.func");
    c.accept("public");
    c.accept("private");
    c.expect("@");
    HFunc f;
    f.name = c.ident();
    c.expect("(");
    if (!c.accept(")")) {
      do {
        f.arg_names.push_back(c.value());
        c.expect(":");
        f.args.push_back(c.type());
        if (c.peek("{")) {  // argument attributes
          int depth = 0;
          const std::string& s = c.str();
          size_t p = c.pos();
          do {
            if (s[p] == '{') depth++;
            if (s[p] == '}') depth--;
            ++p;
          } while (p < s.size() && depth > 0);
          c.set(p);
        }
      } while (c.accept(","));
      c.expect(")");
    }
    c.expect("->");
    f.rets = c.type_list();
    c.expect("{");
    // statements
    while (true) {
      c.ws();
      if (c.accept("}")) break;
      if (c.accept("return") || c.accept("func.return") || c.accept("stablehlo.return")) {
        do f.ret_names.push_back(c.value());
        while (c.accept(","));
        c.expect(":");
        c.type_list();  // return types (repeated)
        while (c.accept(",")) c.type();
        continue;
      }
      // one statement: up to a newline at bracket depth 0 that is followed by
      // the start of the next statement ("%x =", "return" or the closing
      // brace); other lines continue it (the printer may wrap long ops)
      const std::string& s = c.str();
      size_t p = c.pos();
      int depth = 0;
      std::string stmt;
      auto starts_statement = [&](size_t q) {
        while (q < s.size() && (s[q] == ' ' || s[q] == '\t' || s[q] == '\r' || s[q] == '\n')) ++q;
        if (q >= s.size() || s[q] == '}') return true;
        if (s.compare(q, 6, "return") == 0 || s.compare(q, 11, "func.return") == 0) return true;
        // "%x =" or "%x, %y =" (multi-result ops)
        while (true) {
          if (q >= s.size() || s[q] != '%') return false;
          ++q;
          while (q < s.size() && (std::isalnum(static_cast<unsigned char>(s[q])) || s[q] == '_' || s[q] == '#')) ++q;
          while (q < s.size() && s[q] == ' ') ++q;
          if (q < s.size() && s[q] == ',') {
            ++q;
            while (q < s.size() && s[q] == ' ') ++q;
            continue;
          }
          return q < s.size() && s[q] == '=';
        }
      };
      while (p < s.size()) {
        const char ch = s[p];
        if (ch == '{' || ch == '(' || ch == '[') depth++;
        if (ch == '}' || ch == ')' || ch == ']') depth--;
        if (ch == '\n' && depth <= 0 && starts_statement(p + 1)) break;
        stmt += (ch == '\n') ? ' ' : ch;
        ++p;
      }
      c.set(p);
      f.ops.push_back(parse_op(stmt));
    }
    if (f.ret_names.size() != f.rets.size()) c.fail("return arity does not match the signature");
    m.funcs.push_back(std::move(f));
  }
  if (m.name.empty()) m.name = "module";
  return m;
}

// ---------------------------------------------------------------------------
// Generic executor
// ---------------------------------------------------------------------------

struct ValueLoc {
  int kind = 0;        // 0 = arena, 1 = argument, 2 = constant region
  size_t offset = 0;   // arena / constant offset, or argument index
  TType type;
};

float host_bf16(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  if (std::isnan(v)) b = (b | 0x00400000u) & 0xFFFF0000u;
  else b = ((b + 0x7FFFu + ((b >> 16) & 1u)) & 0xFFFF0000u);
  float r;
  std::memcpy(&r, &b, 4);
  return r;
}

class GenericFunc {
 public:
  HFunc f;
  std::map<std::string, ValueLoc> loc;
  std::map<std::string, std::string> root;  // reshape alias root
  size_t arena_bytes = 0, const_bytes = 0, scratch_bytes = 0, scratch_off = 0;
  std::vector<char> const_host;
  char* arena = nullptr;
  char* consts = nullptr;
  bool ready = false;

  ~GenericFunc() {
    if (consts) cudaFree(consts);  // one allocation: constants, then the arena
  }

  static std::vector<int64_t> strides_of(const std::vector<int64_t>& shape) {
    std::vector<int64_t> st(shape.size(), 1);
    for (int i = static_cast<int>(shape.size()) - 2; i >= 0; --i) st[i] = st[i + 1] * shape[i + 1];
    return st;
  }

  std::string rootof(const std::string& v) const {
    auto it = root.find(v);
    return it == root.end() ? v : it->second;
  }

  // Validates every op and plans memory; throws ParseError on anything the
  // executor cannot run.
  void plan() {
    std::map<std::string, TType> types;
    for (size_t i = 0; i < f.args.size(); ++i) {
      const std::string n = "%arg" + std::to_string(i);
      types[n] = f.args[i];
      loc[n] = ValueLoc{1, i, f.args[i]};
    }
    // constants first (host image), reshape aliases, last uses
    std::map<std::string, size_t> last_use;
    for (size_t i = 0; i < f.ops.size(); ++i) {
      HOp& op = f.ops[i];
      for (auto& o : op.operands) {
        if (!types.count(o)) throw ParseError{"use of undefined value " + o + " in: " + op.text};
        last_use[rootof(o)] = i;
      }
      check_op(op, types);
      types[op.result] = op.type;
      if (!op.result2.empty()) types[op.result2] = op.type2;
      if (op.kind == "reshape") root[op.result] = rootof(op.operands[0]);
    }
    for (auto& r : f.ret_names) {
      if (!types.count(r)) throw ParseError{"return of undefined value " + r};
      last_use[rootof(r)] = f.ops.size();
    }
    for (size_t i = 0; i < f.ret_names.size(); ++i) {
      if (!(types[f.ret_names[i]] == f.rets[i])) throw ParseError{"return type mismatch for " + f.ret_names[i]};
      if (f.rets[i].dt == DT_I1) throw ParseError{"boolean function results are not supported"};
    }
    for (auto& a : f.args)
      if (a.dt == DT_I1) throw ParseError{"boolean function arguments are not supported"};
    // constant region
    for (auto& op : f.ops) {
      if (op.kind != "constant") continue;
      const size_t off = (const_host.size() + 255) & ~size_t(255);
      const size_t bytes = op.type.bytes();
      const_host.resize(off + std::max<size_t>(bytes, 1));
      fill_constant(op, const_host.data() + off);
      loc[op.result] = ValueLoc{2, off, op.type};
    }
    const_bytes = (const_host.size() + 255) & ~size_t(255);
    // arena: first-fit over [offset, size) blocks, freed after the last use
    std::vector<std::pair<size_t, size_t>> live;  // offset, size (sorted by offset)
    auto alloc = [&](size_t bytes) {
      bytes = (std::max<size_t>(bytes, 1) + 255) & ~size_t(255);
      size_t off = 0;
      for (auto& b : live) {
        if (b.first >= off + bytes) break;
        off = std::max(off, b.first + b.second);
      }
      live.push_back({off, bytes});
      std::sort(live.begin(), live.end());
      arena_bytes = std::max(arena_bytes, off + bytes);
      return off;
    };
    auto release = [&](size_t off) {
      for (size_t k = 0; k < live.size(); ++k)
        if (live[k].first == off) {
          live.erase(live.begin() + k);
          return;
        }
    };
    std::map<size_t, std::vector<std::string>> frees;  // op index -> roots whose last use it is
    for (auto& kv : last_use) frees[kv.second].push_back(kv.first);
    for (size_t i = 0; i < f.ops.size(); ++i) {
      HOp& op = f.ops[i];
      if (op.kind == "reshape") {
        ValueLoc l = loc[rootof(op.operands[0])];
        l.type = op.type;
        loc[op.result] = l;
      } else if (op.kind != "constant") {
        loc[op.result] = ValueLoc{0, alloc(op.type.bytes()), op.type};
        if (!op.result2.empty()) loc[op.result2] = ValueLoc{0, alloc(op.type2.bytes()), op.type2};
      }
      for (auto& r : frees[i]) {
        auto it = loc.find(r);
        if (it != loc.end() && it->second.kind == 0 && !op_is_result_root(op, r)) release(it->second.offset);
      }
    }
    scratch_bytes = 0;
    for (auto& op : f.ops) scratch_bytes = std::max(scratch_bytes, op_scratch(op));
    scratch_off = (arena_bytes + 255) & ~size_t(255);
    arena_bytes = scratch_off + scratch_bytes;
  }

  bool op_is_result_root(const HOp& op, const std::string& r) const {
    return rootof(op.result) == r || (!op.result2.empty() && op.result2 == r);
  }

  static void fill_constant(const HOp& op, char* dst) {
    const int64_t n = op.type.numel();
    const bool hex = op.dim == 1 && !op.dims.empty();
    const size_t nv = op.values.size();
    if (nv != 1 && static_cast<int64_t>(nv) != n) throw ParseError{"constant size mismatch: " + op.text};
    for (int64_t i = 0; i < n; ++i) {
      const size_t k = nv == 1 ? 0 : static_cast<size_t>(i);
      double v = op.values[k];
      switch (op.type.dt) {
        case DT_F32: {
          float x = static_cast<float>(v);
          if (hex) {
            const uint32_t bits = static_cast<uint32_t>(op.dims[k]);
            std::memcpy(&x, &bits, 4);
          }
          std::memcpy(dst + 4 * i, &x, 4);
          break;
        }
        case DT_BF16: {
          uint16_t b;
          if (hex) {
            b = static_cast<uint16_t>(op.dims[k]);
          } else {
            const float r = host_bf16(static_cast<float>(v));
            uint32_t u;
            std::memcpy(&u, &r, 4);
            b = static_cast<uint16_t>(u >> 16);
          }
          std::memcpy(dst + 2 * i, &b, 2);
          break;
        }
        case DT_F16: {
          if (hex) {
            const uint16_t b = static_cast<uint16_t>(op.dims[k]);
            std::memcpy(dst + 2 * i, &b, 2);
          } else {
            const __half h = __float2half_rn(static_cast<float>(v));
            std::memcpy(dst + 2 * i, &h, 2);
          }
          break;
        }
        case DT_I32: {
          const int32_t x = hex ? static_cast<int32_t>(static_cast<uint32_t>(op.dims[k])) : static_cast<int32_t>(v);
          std::memcpy(dst + 4 * i, &x, 4);
          break;
        }
        default: {
          const uint8_t x = v != 0.0;
          dst[i] = static_cast<char>(x);
        }
      }
    }
  }

  // canonical dot_general description
  struct Dot {
    std::vector<int64_t> lperm, rperm;  // to [batch, free, contract] / [batch, contract, free]
    bool lid = true, rid = true;
    int64_t batch = 1, M = 1, N = 1, K = 1;
  };

  static Dot dot_of(const HOp& op) {
    const auto& ls = op.operand_types[0].shape;
    const auto& rs = op.operand_types[1].shape;
    Dot d;
    std::vector<bool> lused(ls.size()), rused(rs.size());
    for (auto b : op.lb) {
      d.lperm.push_back(b);
      lused[b] = true;
      d.batch *= ls[b];
    }
    for (auto b : op.rb) {
      d.rperm.push_back(b);
      rused[b] = true;
    }
    std::vector<int64_t> lfree, rfree;
    for (size_t i = 0; i < ls.size(); ++i)
      if (!lused[i] && std::find(op.lc.begin(), op.lc.end(), static_cast<int64_t>(i)) == op.lc.end())
        lfree.push_back(i);
    for (size_t i = 0; i < rs.size(); ++i)
      if (!rused[i] && std::find(op.rc.begin(), op.rc.end(), static_cast<int64_t>(i)) == op.rc.end())
        rfree.push_back(i);
    for (auto i : lfree) {
      d.lperm.push_back(i);
      d.M *= ls[i];
    }
    for (auto i : op.lc) {
      d.lperm.push_back(i);
      d.K *= ls[i];
    }
    for (auto i : op.rc) d.rperm.push_back(i);
    for (auto i : rfree) {
      d.rperm.push_back(i);
      d.N *= rs[i];
    }
    for (size_t i = 0; i < d.lperm.size(); ++i)
      if (d.lperm[i] != static_cast<int64_t>(i)) d.lid = false;
    for (size_t i = 0; i < d.rperm.size(); ++i)
      if (d.rperm[i] != static_cast<int64_t>(i)) d.rid = false;
    return d;
  }

  static bool use_library_gemm(const HOp& op, const Dot& d) {
    const int dl = op.operand_types[0].dt, dr = op.operand_types[1].dt, dc = op.type.dt;
    if (d.batch != 1 || dl != dr) return false;
    if (dl == DT_BF16) return (d.K % 8 == 0) && (d.N % 8 == 0) && (dc == DT_BF16 || dc == DT_F32);
    if (dl == DT_F32) return dc == DT_F32;
    return false;
  }

  static GemmDesc gemm_desc(const Dot& d, const void* A, const void* B, void* C, int dc) {
    GemmDesc g;
    g.A = A;
    g.lda = d.K;
    g.a_mn = false;
    g.B = B;
    g.ldb = d.N;
    g.b_mn = true;
    g.M = static_cast<int>(d.M);
    g.N = static_cast<int>(d.N);
    g.K = static_cast<int>(d.K);
    g.out = C;
    g.ldo = d.N;
    g.out_f32 = dc == DT_F32;
    return g;
  }

  size_t op_scratch(const HOp& op) const {
    if (op.kind == "sort") {
      const int64_t len = op.type.shape.back();
      return len ? sort_rows_workspace_bytes(op.type.numel() / len, static_cast<int>(len)) : 0;
    }
    if (op.kind != "dot_general") return 0;
    Dot d = dot_of(op);
    size_t s = 0;
    if (!d.lid) s += (op.operand_types[0].bytes() + 255) & ~size_t(255);
    if (!d.rid) s += (op.operand_types[1].bytes() + 255) & ~size_t(255);
    if (use_library_gemm(op, d)) {
      GemmDesc g = gemm_desc(d, nullptr, nullptr, nullptr, op.type.dt);
      s += gemm_workspace_bytes(g, op.operand_types[0].dt == DT_BF16);
    }
    return s;
  }

  static void check_op(HOp& op, const std::map<std::string, TType>& types) {
    // fill operand types from the SSA environment where the printer omits them
    if (op.operand_types.size() != op.operands.size()) {
      op.operand_types.clear();
      for (auto& o : op.operands) op.operand_types.push_back(types.at(o));
    } else {
      for (size_t i = 0; i < op.operands.size(); ++i)
        if (!(types.at(op.operands[i]) == op.operand_types[i]))
          throw ParseError{"operand type mismatch in: " + op.text};
    }
    if (op.type.shape.size() > static_cast<size_t>(kMaxRank)) throw ParseError{"rank above 8: " + op.text};
    const auto& k = op.kind;
    if (k == "unary" || k == "binary" || k == "compare" || k == "convert" || k == "clamp" || k == "select") {
      // elementwise: every non-scalar operand has the result's shape
      for (size_t i = 0; i < op.operand_types.size(); ++i) {
        const bool scalar_ok = (k == "clamp" && i != 1) || (k == "select" && i == 0);
        const auto& s = op.operand_types[i].shape;
        if (!(s == op.type.shape) && !(scalar_ok && s.empty()))
          throw ParseError{"elementwise shape mismatch: " + op.text};
      }
      if ((k == "binary" || k == "unary" || k == "clamp") && op.operand_types[k == "clamp" ? 1 : 0].dt != op.type.dt)
        throw ParseError{"elementwise element type mismatch: " + op.text};
      if (k == "compare" && op.type.dt != DT_I1) throw ParseError{"compare must produce i1: " + op.text};
    }
    auto i32_scalars_from = [&](size_t first) {
      for (size_t i = first; i < op.operand_types.size(); ++i)
        if (op.operand_types[i].dt != DT_I32 || !op.operand_types[i].shape.empty())
          throw ParseError{"start indices must be i32 scalars: " + op.text};
    };
    if (k == "reverse") {
      for (auto d : op.dims)
        if (d < 0 || d >= static_cast<int64_t>(op.type.shape.size())) throw ParseError{"reverse dimension: " + op.text};
      if (!(op.type == op.operand_types[0])) throw ParseError{"reverse type mismatch: " + op.text};
    } else if (k == "dynamic_slice") {
      const auto& sh = op.operand_types[0].shape;
      if (op.operands.size() != 1 + sh.size() || op.slice_sizes.size() != sh.size())
        throw ParseError{"dynamic_slice needs one start index per dimension: " + op.text};
      i32_scalars_from(1);
      for (size_t d = 0; d < sh.size(); ++d)
        if (op.slice_sizes[d] < 0 || op.slice_sizes[d] > sh[d]) throw ParseError{"dynamic_slice size: " + op.text};
      if (op.type.shape != op.slice_sizes || op.type.dt != op.operand_types[0].dt)
        throw ParseError{"dynamic_slice result type: " + op.text};
    } else if (k == "dynamic_update_slice") {
      const auto& sh = op.operand_types[0].shape;
      if (op.operands.size() != 2 + sh.size()) throw ParseError{"dynamic_update_slice arity: " + op.text};
      const TType& u = op.operand_types[1];
      if (u.shape.size() != sh.size() || u.dt != op.operand_types[0].dt)
        throw ParseError{"dynamic_update_slice update type: " + op.text};
      for (size_t d = 0; d < sh.size(); ++d)
        if (u.shape[d] > sh[d]) throw ParseError{"dynamic_update_slice update larger than operand: " + op.text};
      i32_scalars_from(2);
      if (!(op.type == op.operand_types[0])) throw ParseError{"dynamic_update_slice result type: " + op.text};
    } else if (k == "sort") {
      const TType& kt = op.operand_types.at(0);
      const TType& pt = op.operand_types.at(1);
      if (op.operands.size() != 2 || kt.shape != pt.shape || kt.shape.empty())
        throw ParseError{"sort takes keys and a payload of one shape: " + op.text};
      if ((kt.dt != DT_F32 && kt.dt != DT_BF16) || pt.dt != DT_I32)
        throw ParseError{"sort keys must be f32 or bf16 and the payload i32: " + op.text};
      if (op.dim != static_cast<int64_t>(kt.shape.size()) - 1) throw ParseError{"sort along the last axis only: " + op.text};
      if (kt.shape.back() > kSortMaxRow)
        throw ParseError{"sort rows longer than " + std::to_string(kSortMaxRow) + ": " + op.text};
      if (!(op.type == kt) || !(op.type2 == pt)) throw ParseError{"sort result types: " + op.text};
    }
    if (k == "pad") {
      for (auto v : op.interior)
        if (v != 0) throw ParseError{"interior padding is not supported: " + op.text};
      for (auto v : op.low)
        if (v < 0) throw ParseError{"negative padding is not supported: " + op.text};
    } else if (k == "reduce") {
      auto dims = op.dims;
      std::sort(dims.begin(), dims.end());
      for (size_t i = 1; i < dims.size(); ++i)
        if (dims[i] != dims[i - 1] + 1) throw ParseError{"reduce over non-adjacent dimensions: " + op.text};
    } else if (k == "gather") {
      const auto& os = op.operand_types[0].shape;
      const auto& is = op.operand_types[1].shape;
      const bool ok = op.collapsed == std::vector<int64_t>{0} && op.start_index_map == std::vector<int64_t>{0} &&
                      op.operand_batching.empty() && !is.empty() && is.back() == 1 &&
                      op.index_vector_dim == static_cast<int64_t>(is.size()) - 1 &&
                      op.operand_types[1].dt == DT_I32 && op.slice_sizes.size() == os.size() &&
                      op.slice_sizes[0] == 1;
      if (!ok) throw ParseError{"only row gathers (collapsed_slice_dims = [0]) are supported: " + op.text};
      for (size_t i = 1; i < os.size(); ++i)
        if (op.slice_sizes[i] != os[i]) throw ParseError{"partial-row gather is not supported: " + op.text};
    }
  }

  sb_status init(Session& s) {
    if (ready) return nullptr;
    void* p = nullptr;
    if (cudaMalloc(&p, const_bytes + arena_bytes + 256) != cudaSuccess)
      return make_status(SB_STATUS_RESOURCE_EXHAUSTED, "module arena allocation failed");
    consts = static_cast<char*>(p);
    arena = consts + const_bytes;
    if (!const_host.empty())
      SB_CUDA_TRY(cudaMemcpyAsync(consts, const_host.data(), const_host.size(), cudaMemcpyHostToDevice, s.stream));
    ready = true;
    return nullptr;
  }

  void* ptr(const std::string& v, const std::vector<Buffer*>& in) const {
    const ValueLoc& l = loc.at(v);
    if (l.kind == 1) return in[l.offset]->data();
    if (l.kind == 2) return consts + l.offset;
    return arena + l.offset;
  }

  sb_status run(Session& s, const std::vector<Buffer*>& in, std::vector<Buffer*>& out) {
    SB_TRY(init(s));
    SB_RETURN_IF(in.size() != f.args.size(), SB_STATUS_INVALID_ARGUMENT,
                 f.name + " expects " + std::to_string(f.args.size()) + " inputs, got " + std::to_string(in.size()));
    for (size_t i = 0; i < in.size(); ++i) {
      SB_RETURN_IF(in[i]->shape != f.args[i].shape || in[i]->elem != elem_of(f.args[i].dt),
                   SB_STATUS_INVALID_ARGUMENT, "input " + std::to_string(i) + " does not match the signature");
    }
    cudaStream_t st = s.stream;
    for (const HOp& op : f.ops) {
      int rc = exec(op, in, st, s.err_word);
      if (rc) return make_status(SB_STATUS_INTERNAL, "kernel launch failed (" + std::to_string(rc) + ") in: " + op.text);
    }
    size_t total = 0;
    std::vector<size_t> offs;
    for (auto& r : f.rets) {
      offs.push_back(total);
      total = (total + std::max<size_t>(r.bytes(), 1) + 255) & ~size_t(255);
    }
    Allocation* a = nullptr;
    SB_TRY(session_alloc(s, total, &a));
    a->refs.store(static_cast<int>(f.rets.size()));
    for (size_t i = 0; i < f.rets.size(); ++i) {
      if (f.rets[i].bytes())
        SB_CUDA_TRY(cudaMemcpyAsync(static_cast<char*>(a->ptr) + offs[i], ptr(f.ret_names[i], in), f.rets[i].bytes(),
                                    cudaMemcpyDeviceToDevice, st));
      out.push_back(buffer_new(s, a, offs[i], f.rets[i].shape, elem_of(f.rets[i].dt)));
    }
    s.kernel_launches += f.ops.size();
    return nullptr;
  }

  int exec(const HOp& op, const std::vector<Buffer*>& in, cudaStream_t st, int* err) {
    const auto& k = op.kind;
    void* o = (k == "constant") ? nullptr : ptr(op.result, in);
    const long n = op.type.numel();
    auto P = [&](int i) { return ptr(op.operands[i], in); };
    if (k == "constant" || k == "reshape") return 0;
    if (k == "unary") return unary(P(0), o, n, op.unary_op, op.operand_types[0].dt, op.type.dt, st);
    if (k == "binary") return binary(P(0), P(1), o, n, op.binary_op, op.type.dt, st);
    if (k == "convert") return convert(P(0), op.operand_types[0].dt, o, op.type.dt, n, st);
    if (k == "clamp")
      return clamp(P(0), op.operand_types[0].numel(), P(1), P(2), op.operand_types[2].numel(), o, n, op.type.dt, st);
    if (k == "compare") return compare(P(0), P(1), o, n, op.cmp, op.operand_types[0].dt, st);
    if (k == "select") return select(P(0), op.operand_types[0].numel(), P(1), P(2), o, n, op.type.dt, st);
    if (k == "iota") {
      long inner = 1;
      for (size_t i = op.dim + 1; i < op.type.shape.size(); ++i) inner *= op.type.shape[i];
      return iota(o, n, op.type.dt, inner, op.type.shape.empty() ? 1 : op.type.shape[op.dim], st);
    }
    if (k == "broadcast_in_dim" || k == "transpose" || k == "slice" || k == "pad") {
      const auto& is = op.operand_types[0].shape;
      const auto ist = strides_of(is);
      IndexMap m;
      m.rank = static_cast<int>(op.type.shape.size());
      for (int d = 0; d < m.rank; ++d) m.out_shape[d] = op.type.shape[d];
      if (k == "broadcast_in_dim") {
        for (size_t i = 0; i < op.dims.size(); ++i)
          if (is[i] != 1) m.stride[op.dims[i]] = ist[i];
      } else if (k == "transpose") {
        for (int d = 0; d < m.rank; ++d) m.stride[d] = ist[op.dims[d]];
      } else if (k == "slice") {
        for (int d = 0; d < m.rank; ++d) {
          m.stride[d] = ist[d] * op.strides[d];
          m.base += op.starts[d] * ist[d];
        }
      } else {
        m.check = true;
        m.pad_value = P(1);
        for (int d = 0; d < m.rank; ++d) {
          m.stride[d] = ist[d];
          m.offset[d] = op.low[d];
          m.extent[d] = is[d];
        }
      }
      if (m.rank == 0) {
        m.rank = 1;
        m.out_shape[0] = 1;
      }
      return remap(P(0), o, n, op.type.dt, m, st);
    }
    if (k == "reverse") {
      const auto& sh = op.type.shape;
      const auto ist = strides_of(sh);
      IndexMap m;
      m.rank = static_cast<int>(sh.size());
      for (int d = 0; d < m.rank; ++d) {
        m.out_shape[d] = sh[d];
        m.stride[d] = ist[d];
      }
      for (auto d : op.dims) {
        m.base += (sh[d] - 1) * ist[d];
        m.stride[d] = -ist[d];
      }
      if (m.rank == 0) {
        m.rank = 1;
        m.out_shape[0] = 1;
      }
      return remap(P(0), o, n, op.type.dt, m, st);
    }
    if (k == "dynamic_slice" || k == "dynamic_update_slice") {
      const bool upd = k == "dynamic_update_slice";
      const auto& sh = op.operand_types[0].shape;
      DynSlice d;
      d.rank = static_cast<int>(sh.size());
      for (int a = 0; a < d.rank; ++a) {
        d.shape[a] = sh[a];
        d.size[a] = upd ? op.operand_types[1].shape[a] : op.slice_sizes[a];
        d.start[a] = static_cast<const int32_t*>(P((upd ? 2 : 1) + a));
      }
      if (!upd) return dynamic_slice(P(0), o, op.type.dt, d, st);
      if (o != P(0) && op.type.bytes() &&
          cudaMemcpyAsync(o, P(0), op.type.bytes(), cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return 4;
      return dynamic_update(o, P(1), op.type.dt, d, st);
    }
    if (k == "sort") {
      const int len = static_cast<int>(op.type.shape.back());
      const long rows = len ? n / len : 0;
      return sort_rows(P(0), op.type.dt, static_cast<const int32_t*>(P(1)), o, static_cast<int32_t*>(ptr(op.result2, in)),
                       rows, len, op.descending, arena + scratch_off, sort_rows_workspace_bytes(rows, len), st);
    }
    if (k == "concatenate") {
      long off = 0;
      for (size_t j = 0; j < op.operands.size(); ++j) {
        const auto& is = op.operand_types[j].shape;
        const auto ist = strides_of(is);
        IndexMap m;
        m.rank = static_cast<int>(op.type.shape.size());
        m.check = true;
        for (int d = 0; d < m.rank; ++d) {
          m.out_shape[d] = op.type.shape[d];
          m.stride[d] = ist[d];
          m.extent[d] = is[d];
          m.offset[d] = (d == op.dim) ? off : 0;
        }
        int rc = remap(P(static_cast<int>(j)), o, n, op.type.dt, m, st);
        if (rc) return rc;
        off += is[op.dim];
      }
      return 0;
    }
    if (k == "reduce") {
      const auto& is = op.operand_types[0].shape;
      auto dims = op.dims;
      std::sort(dims.begin(), dims.end());
      long outer = 1, red = 1, inner = 1;
      for (size_t i = 0; i < is.size(); ++i) {
        if (!dims.empty() && static_cast<int64_t>(i) < dims.front()) outer *= is[i];
        else if (!dims.empty() && static_cast<int64_t>(i) > dims.back()) inner *= is[i];
        else if (!dims.empty()) red *= is[i];
        else outer *= is[i];
      }
      return reduce(P(0), o, outer, red, inner, op.reduce_op, 0.f, P(1), op.type.dt, st);
    }
    if (k == "gather") {
      const auto& os = op.operand_types[0].shape;
      long width = 1;
      for (size_t i = 1; i < os.size(); ++i) width *= os[i];
      return gather_rows(P(0), P(1), o, op.operand_types[1].numel(), os[0], width, op.type.dt, st);
    }
    if (k == "dot_general") {
      Dot d = dot_of(op);
      char* scratch = arena + scratch_off;
      const void* A = P(0);
      const void* B = P(1);
      auto permute = [&](const TType& t, const std::vector<int64_t>& perm, const void* src, char* dst) {
        const auto ist = strides_of(t.shape);
        IndexMap m;
        m.rank = static_cast<int>(t.shape.size());
        for (int dd = 0; dd < m.rank; ++dd) {
          m.out_shape[dd] = t.shape[perm[dd]];
          m.stride[dd] = ist[perm[dd]];
        }
        return remap(src, dst, t.numel(), t.dt, m, st);
      };
      if (!d.lid) {
        if (int rc = permute(op.operand_types[0], d.lperm, A, scratch)) return rc;
        A = scratch;
        scratch += (op.operand_types[0].bytes() + 255) & ~size_t(255);
      }
      if (!d.rid) {
        if (int rc = permute(op.operand_types[1], d.rperm, B, scratch)) return rc;
        B = scratch;
        scratch += (op.operand_types[1].bytes() + 255) & ~size_t(255);
      }
      if (use_library_gemm(op, d)) {
        GemmDesc g = gemm_desc(d, A, B, o, op.type.dt);
        const bool bf = op.operand_types[0].dt == DT_BF16;
        const size_t ws = gemm_workspace_bytes(g, bf);
        return bf ? gemm_bf16(g, reinterpret_cast<float*>(scratch), ws, st, err)
                  : gemm_f32(g, reinterpret_cast<float*>(scratch), ws, st, err);
      }
      return bgemm(A, B, o, static_cast<int>(d.batch), static_cast<int>(d.M), static_cast<int>(d.N),
                   static_cast<int>(d.K), op.operand_types[0].dt, op.operand_types[1].dt, op.type.dt, st);
    }
    return 1;
  }
};

// ---------------------------------------------------------------------------
// Recognizer: nanoGPT value_and_grad
// ---------------------------------------------------------------------------

bool match_gpt_vag(const HFunc& f, GptShape* g) {
  if (f.name.find("value_and_grad") == std::string::npos) return false;
  const size_t na = f.args.size();
  if (na < 12 || (na - 6) % 6 != 0) return false;
  const int L = static_cast<int>((na - 6) / 6);
  const int dt = f.args[0].dt;
  if (dt != DT_BF16 && dt != DT_F32) return false;
  const auto& head = f.args[0].shape;
  if (head.size() != 2) return false;
  const int64_t V = head[0], D = head[1];
  auto is = [&](size_t i, std::vector<int64_t> s) { return f.args[i].dt == dt && f.args[i].shape == s; };
  for (int l = 0; l < L; ++l) {
    const size_t b = 1 + 6 * l;
    if (!is(b, {3 * D, D}) || !is(b + 1, {D, D}) || !is(b + 2, {D}) || !is(b + 3, {D}) || !is(b + 4, {4 * D, D}) ||
        !is(b + 5, {D, 4 * D}))
      return false;
  }
  const size_t t = 1 + 6 * L;
  if (!is(t, {D}) || f.args[t + 1].dt != dt || f.args[t + 1].shape.size() != 2 || f.args[t + 1].shape[1] != D ||
      !is(t + 2, {V, D}))
    return false;
  const int64_t P = f.args[t + 1].shape[0];
  const TType& x = f.args[t + 3];
  const TType& y = f.args[t + 4];
  if (x.dt != DT_F32 || !(x == y) || x.shape.size() != 2) return false;
  const int64_t B = x.shape[0], T = x.shape[1];
  if (T > P) return false;
  if (f.rets.size() != 1 + t + 3 || !f.rets[0].shape.empty() || f.rets[0].dt != dt) return false;
  for (size_t i = 0; i <= t + 2; ++i)
    if (!(f.rets[1 + i] == f.args[i])) return false;
  // heads: the q/k/v split reshapes [B*T or B, T, D] into [B, T, H, D/H]
  int H = 0;
  int gathers = 0, dots = 0;
  for (auto& op : f.ops) {
    if (op.kind == "gather" && op.operand_types[0].shape == std::vector<int64_t>({V, D})) ++gathers;
    if (op.kind == "dot_general") ++dots;
    const auto& s = op.type.shape;
    if (op.kind == "reshape" && s.size() == 4 && s[0] == B && s[1] == T && s[2] * s[3] == D && H == 0)
      H = static_cast<int>(s[2]);
  }
  if (H == 0 || gathers < 1 || dots < 4 * L) return false;
  *g = GptShape{L, H, static_cast<int>(D), static_cast<int>(P), static_cast<int>(V), static_cast<int>(B),
                static_cast<int>(T), elem_of(dt)};
  return true;
}

// The nanoGPT params leaves (sorted keys: lm_head, the blocks' six leaves each,
// ln_f, wpe, wte) as args[first .. first + n) of element type dt; sets the
// layer count, vocabulary, width and wpe rows.
bool gpt_leaf_layout(const std::vector<TType>& a, size_t first, size_t n, int dt, int* L_out, int64_t* V_out,
                     int64_t* D_out, int64_t* P_out) {
  if (n < 10 || (n - 4) % 6 != 0 || first + n > a.size()) return false;
  const int L = static_cast<int>((n - 4) / 6);
  const auto& head = a[first].shape;
  if (a[first].dt != dt || head.size() != 2) return false;
  const int64_t V = head[0], D = head[1];
  auto is = [&](size_t i, std::vector<int64_t> sh) { return a[first + i].dt == dt && a[first + i].shape == sh; };
  for (int l = 0; l < L; ++l) {
    const size_t b = 1 + 6 * l;
    if (!is(b, {3 * D, D}) || !is(b + 1, {D, D}) || !is(b + 2, {D}) || !is(b + 3, {D}) || !is(b + 4, {4 * D, D}) ||
        !is(b + 5, {D, 4 * D}))
      return false;
  }
  const size_t t = 1 + 6 * L;
  const TType& wpe = a[first + t + 1];
  if (!is(t, {D}) || wpe.dt != dt || wpe.shape.size() != 2 || wpe.shape[1] != D || !is(t + 2, {V, D})) return false;
  *L_out = L;
  *V_out = V;
  *D_out = D;
  *P_out = wpe.shape[0];
  return true;
}

// Heads of the attention: the q/k/v split reshapes [.., T, D] into [B, T, H, D/H].
int gpt_heads(const HFunc& f, int64_t B, int64_t T, int64_t V, int64_t D, int L) {
  int H = 0, gathers = 0, dots = 0;
  for (auto& op : f.ops) {
    if (op.kind == "gather" && op.operand_types[0].shape == std::vector<int64_t>({V, D})) ++gathers;
    if (op.kind == "dot_general") ++dots;
    const auto& s = op.type.shape;
    if (op.kind == "reshape" && s.size() == 4 && s[0] == B && s[1] == T && s[2] * s[3] == D && H == 0)
      H = static_cast<int>(s[2]);
  }
  return (gathers >= 1 && dots >= 4 * L) ? H : 0;
}

// Recognizer: nanoGPT train-step (examples/nanogpt/train.shf:26-33), one
// module holding value_and_grad, clip-by-global-norm and adamw-step
// (lib/optim.shf). Arguments: the state pytree's leaves in sorted-key order
// -- an optional key [4] (f32), loss, m leaves, params leaves, t (f32), v
// leaves -- then x, y (f32 ids [B, T]) and lr (f32); results: the new state
// in the same order. The hyperparameters are literals in the module; they are
// read off the ops that use them: b1 and b2 multiply the incoming m and v,
// wd the incoming params, eps is added to sqrt(v-hat), and max_norm divides
// the global norm plus 1e-8.
bool match_gpt_train(const HFunc& f, GptShape* g, AdamwConfig* hp, bool* has_key) {
  if (f.name.find("train_step") == std::string::npos) return false;
  const size_t na = f.args.size();
  for (size_t k = 0; k <= 1; ++k) {
    if (k == 1 && !(f.args[0].dt == DT_F32 && f.args[0].shape == std::vector<int64_t>({4}))) continue;
    if (na < k + 5 || (na - k - 5) % 3 != 0) continue;
    const size_t n = (na - k - 5) / 3;
    const int dt = f.args[k].dt;
    if ((dt != DT_BF16 && dt != DT_F32) || !f.args[k].shape.empty()) continue;
    int L = 0;
    int64_t V = 0, D = 0, P = 0;
    const size_t im = k + 1, ip = k + 1 + n, it = k + 1 + 2 * n, iv = k + 2 + 2 * n, ix = k + 2 + 3 * n;
    if (!gpt_leaf_layout(f.args, ip, n, dt, &L, &V, &D, &P)) continue;
    bool same = true;
    for (size_t i = 0; i < n; ++i) same = same && f.args[im + i] == f.args[ip + i] && f.args[iv + i] == f.args[ip + i];
    const TType& t = f.args[it];
    const TType& x = f.args[ix];
    const TType& lr = f.args[ix + 2];
    if (!same || t.dt != DT_F32 || !t.shape.empty() || lr.dt != DT_F32 || !lr.shape.empty()) continue;
    if (x.dt != DT_F32 || !(x == f.args[ix + 1]) || x.shape.size() != 2 || x.shape[1] > P) continue;
    if (f.rets.size() != ix) continue;
    bool rets_ok = true;
    for (size_t i = 0; i < ix; ++i) rets_ok = rets_ok && f.rets[i] == f.args[i];
    if (!rets_ok) continue;
    const int64_t B = x.shape[0], T = x.shape[1];
    const int H = gpt_heads(f, B, T, V, D, L);
    if (H == 0) continue;
    // hyperparameters
    std::map<std::string, const HOp*> def;
    for (auto& op : f.ops) def[op.result] = &op;
    std::function<bool(const std::string&, double*)> scalar = [&](const std::string& r, double* v) {
      auto it2 = def.find(r);
      if (it2 == def.end()) return false;
      const HOp* op = it2->second;
      if (op->kind == "constant") {
        if (op->values.size() != 1) return false;
        *v = op->values[0];
        return true;
      }
      if (op->kind == "broadcast_in_dim" || op->kind == "convert" || op->kind == "reshape")
        return scalar(op->operands[0], v);
      return false;
    };
    auto bin = [](const HOp& op, int b) { return op.kind == "binary" && op.binary_op == b && op.operands.size() == 2; };
    auto is_sqrt = [&](const std::string& r) {
      auto it2 = def.find(r);
      return it2 != def.end() && it2->second->kind == "unary" && it2->second->unary_op == U_SQRT;
    };
    // the constant operand of a multiply whose other operand is `r`
    auto const_times = [&](const std::string& r, double* v) {
      for (auto& op : f.ops)
        if (bin(op, B_MUL))
          for (int s2 = 0; s2 < 2; ++s2)
            if (op.operands[s2] == r && scalar(op.operands[1 - s2], v)) return true;
      return false;
    };
    double b1 = 0, b2 = 0, wd = 0, eps = 0, mx = 0;
    bool found_eps = false, found_mx = false;
    for (auto& op : f.ops) {
      if (bin(op, B_ADD) && op.type.shape == f.args[ip].shape)
        for (int s2 = 0; s2 < 2 && !found_eps; ++s2)
          if (is_sqrt(op.operands[s2]) && scalar(op.operands[1 - s2], &eps)) found_eps = true;
      if (bin(op, B_DIV) && op.type.shape.empty() && !found_mx) {
        double c = 0;
        auto d = def.find(op.operands[1]);
        if (scalar(op.operands[0], &mx) && d != def.end() && bin(*d->second, B_ADD) &&
            (scalar(d->second->operands[1], &c) || scalar(d->second->operands[0], &c)) &&
            std::fabs(c - 1e-8) < 1e-12)
          found_mx = true;
      }
    }
    if (f.arg_names.size() != na || !const_times(f.arg_names[im], &b1) || !const_times(f.arg_names[iv], &b2) ||
        !const_times(f.arg_names[ip], &wd) || !found_eps || !found_mx)
      continue;
    *g = GptShape{L, H, static_cast<int>(D), static_cast<int>(P), static_cast<int>(V), static_cast<int>(B),
                  static_cast<int>(T), elem_of(dt)};
    *hp = AdamwConfig{static_cast<float>(b1), static_cast<float>(b2), static_cast<float>(eps),
                      static_cast<float>(wd), static_cast<float>(mx)};
    *has_key = k == 1;
    return true;
  }
  return false;
}

// Host-side comparison of two output lists (per tensor, relative to the
// largest magnitude of the reference). *worst receives the largest
// max|a - b| / max|b| over the tensors.
sb_status outputs_agree(const std::vector<Buffer*>& a, const std::vector<Buffer*>& b, double tol, bool* agree,
                        std::string* why, double* worst) {
  *worst = 0;
  *agree = a.size() == b.size();
  for (size_t i = 0; i < a.size() && *agree; ++i) {
    const size_t n = a[i]->bytes();
    if (n != b[i]->bytes() || a[i]->elem != b[i]->elem) {
      *agree = false;
      break;
    }
    std::vector<char> ha(n), hb(n);
    SB_CUDA_TRY(cudaMemcpy(ha.data(), a[i]->data(), n, cudaMemcpyDeviceToHost));
    SB_CUDA_TRY(cudaMemcpy(hb.data(), b[i]->data(), n, cudaMemcpyDeviceToHost));
    const bool bf = a[i]->elem == SB_ELEM_BF16;
    const size_t cnt = n / (bf ? 2 : 4);
    double mx = 0, err = 0;
    for (size_t k = 0; k < cnt; ++k) {
      float va, vb;
      if (bf) {
        uint32_t ua = static_cast<uint32_t>(reinterpret_cast<uint16_t*>(ha.data())[k]) << 16;
        uint32_t ub = static_cast<uint32_t>(reinterpret_cast<uint16_t*>(hb.data())[k]) << 16;
        std::memcpy(&va, &ua, 4);
        std::memcpy(&vb, &ub, 4);
      } else {
        va = reinterpret_cast<float*>(ha.data())[k];
        vb = reinterpret_cast<float*>(hb.data())[k];
      }
      if (!std::isfinite(va)) {
        *agree = false;
        break;
      }
      mx = std::max(mx, std::fabs(static_cast<double>(vb)));
      err = std::max(err, std::fabs(static_cast<double>(va) - vb));
    }
    const double rel = err / std::max(mx, 1e-30);
    *worst = std::max(*worst, rel);
    if (*agree && err > tol * mx) {
      *agree = false;
      *why = "output " + std::to_string(i) + ": max error " + std::to_string(err) + " vs max |ref| " +
             std::to_string(mx);
    }
  }
  return nullptr;
}

// Host copy of a float buffer (f32 or bf16) as doubles.
sb_status host_values(const Buffer* b, std::vector<double>* out) {
  const size_t n = b->bytes();
  std::vector<char> h(n);
  if (n) SB_CUDA_TRY(cudaMemcpy(h.data(), b->data(), n, cudaMemcpyDeviceToHost));
  const bool bf = b->elem == SB_ELEM_BF16;
  const size_t cnt = n / (bf ? 2 : 4);
  out->resize(cnt);
  for (size_t k = 0; k < cnt; ++k) {
    float v;
    if (bf) {
      const uint32_t u = static_cast<uint32_t>(reinterpret_cast<uint16_t*>(h.data())[k]) << 16;
      std::memcpy(&v, &u, 4);
    } else {
      v = reinterpret_cast<float*>(h.data())[k];
    }
    (*out)[k] = v;
  }
  return nullptr;
}

// The first-call comparison of a train step's new state (fast) with the
// generic executor's (ref). loss and m within tol of their largest
// magnitude, v within 2 tol, t exact; parameters by the bound an AdamW step
// allows: p' - p = -lr (wd p + m_hat / (sqrt(v_hat) + eps)), whose Adam part is
// close to lr * sign(g) where v_hat is dominated by g^2, so wherever a gradient
// lies within its own rounding of zero the two results may differ by up to
// 2 lr. Every parameter within 3 lr (plus two ulps of the element type), and
// at most 2% of them beyond 1% of lr.
sb_status train_outputs_agree(const std::vector<Buffer*>& fast, const std::vector<Buffer*>& ref, size_t first,
                              size_t n, double lr, double tol, bool* agree, std::string* why, double* worst) {
  *agree = fast.size() == ref.size() && ref.size() == first + 3 * n + 2;
  *worst = 0;
  if (!*agree) {
    *why = "output count";
    return nullptr;
  }
  size_t flips = 0, total = 0;
  for (size_t i = 0; i < ref.size() && *agree; ++i) {
    std::vector<double> a, b;
    SB_TRY(host_values(fast[i], &a));
    SB_TRY(host_values(ref[i], &b));
    if (a.size() != b.size()) {
      *agree = false;
      *why = "output " + std::to_string(i) + ": size";
      break;
    }
    const size_t j = i - first;  // position in [loss | m | p | t | v]
    if (i < first) {  // the key leaf: passed through
      for (size_t k = 0; k < a.size() && *agree; ++k) *agree = a[k] == b[k];
      if (!*agree) *why = "key leaf";
      continue;
    }
    const bool is_p = j >= 1 + n && j < 1 + 2 * n;
    const bool is_t = j == 1 + 2 * n;
    const bool is_v = j > 1 + 2 * n;
    const bool bf = ref[i]->elem == SB_ELEM_BF16;
    double mx = 0, err = 0;
    for (size_t k = 0; k < a.size(); ++k) {
      if (!std::isfinite(a[k])) {
        *agree = false;
        *why = "output " + std::to_string(i) + ": non-finite";
        break;
      }
      const double d = std::fabs(a[k] - b[k]);
      mx = std::max(mx, std::fabs(b[k]));
      err = std::max(err, d);
      if (is_p) {
        const double slack = std::fabs(b[k]) * (bf ? 1.0 / 128 : 1e-6);
        if (d > 3.0 * lr + slack) {
          *agree = false;
          *why = "parameter output " + std::to_string(i) + ": moved " + std::to_string(d) + " from the reference";
          break;
        }
        if (d > 1e-2 * lr + slack) ++flips;
        ++total;
      }
    }
    if (!*agree) break;
    if (is_t) {
      *agree = err == 0;
      if (!*agree) *why = "t differs";
    } else if (!is_p) {
      const double lim = (is_v ? 2 : 1) * tol;
      *worst = std::max(*worst, err / std::max(mx, 1e-30));
      if (err > lim * mx) {
        *agree = false;
        *why = "output " + std::to_string(i) + ": max error " + std::to_string(err) + " vs max |ref| " +
               std::to_string(mx);
      }
    }
  }
  if (*agree && flips > total / 50) {
    *agree = false;
    *why = std::to_string(flips) + " of " + std::to_string(total) + " parameters differ by more than 1% of lr";
  }
  return nullptr;
}

// ---------------------------------------------------------------------------
// Plan cache (manifest of first-call verification outcomes)
// ---------------------------------------------------------------------------

uint64_t fnv1a(const void* data, size_t n, uint64_t h = 1469598103934665603ull) {
  const unsigned char* p = static_cast<const unsigned char*>(data);
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= 1099511628211ull;
  }
  return h;
}

std::string hex64(uint64_t v) {
  char b[17];
  std::snprintf(b, sizeof b, "%016llx", static_cast<unsigned long long>(v));
  return b;
}

// Hash of the loaded library file: any rebuild invalidates recorded plans.
const std::string& library_id() {
  static const std::string id = [] {
    Dl_info info{};
    if (!dladdr(reinterpret_cast<void*>(&fnv1a), &info) || !info.dli_fname) return std::string("unknown");
    std::ifstream f(info.dli_fname, std::ios::binary);
    if (!f) return std::string("unknown");
    std::string bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    return hex64(fnv1a(bytes.data(), bytes.size()));
  }();
  return id;
}

std::string plan_cache_dir() {
  const char* e = std::getenv("SHEAF_B200_CACHE_DIR");
  return (e && *e) ? std::string(e) : std::string();
}

struct PlanRecord {
  std::string hash, plan, note;
};
using Manifest = std::map<std::string, PlanRecord>;

std::mutex& manifest_mu() {
  static std::mutex mu;
  return mu;
}

std::string json_escape(const std::string& v) {
  std::string o;
  for (char ch : v) {
    if (ch == '"' || ch == '\\') o += '\\';
    if (static_cast<unsigned char>(ch) < 0x20) continue;
    o += ch;
  }
  return o;
}

// Reads the manifest this library writes: {"format": 1, "entries": {"<key>":
// {"hash": "...", "plan": "...", "note": "..."}, ...}}. Anything else reads as
// an empty manifest.
Manifest read_manifest(const std::string& dir) {
  Manifest m;
  std::ifstream f(dir + "/manifest.json");
  if (!f) return m;
  const std::string t((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
  size_t p = 0;
  auto ws = [&]() {
    while (p < t.size() && std::isspace(static_cast<unsigned char>(t[p]))) ++p;
  };
  auto str = [&](std::string* out) {
    ws();
    if (p >= t.size() || t[p] != '"') return false;
    ++p;
    std::string v;
    while (p < t.size() && t[p] != '"') {
      if (t[p] == '\\' && p + 1 < t.size()) ++p;
      v += t[p++];
    }
    if (p >= t.size()) return false;
    ++p;
    *out = v;
    return true;
  };
  auto lit = [&](char ch) {
    ws();
    if (p < t.size() && t[p] == ch) {
      ++p;
      return true;
    }
    return false;
  };
  std::string key;
  if (!lit('{') || !str(&key) || key != "format" || !lit(':')) return {};
  ws();
  while (p < t.size() && std::isdigit(static_cast<unsigned char>(t[p]))) ++p;
  if (!lit(',') || !str(&key) || key != "entries" || !lit(':') || !lit('{')) return {};
  if (lit('}')) return m;
  do {
    std::string name;
    PlanRecord r;
    if (!str(&name) || !lit(':') || !lit('{')) return {};
    do {
      std::string k, v;
      if (!str(&k) || !lit(':') || !str(&v)) return {};
      if (k == "hash") r.hash = v;
      else if (k == "plan") r.plan = v;
      else if (k == "note") r.note = v;
    } while (lit(','));
    if (!lit('}')) return {};
    m[name] = r;
  } while (lit(','));
  return m;
}

// Records one entry (read-modify-write, replaced atomically by rename).
void record_plan(const std::string& dir, const std::string& name, const PlanRecord& r) {
  if (dir.empty()) return;
  std::lock_guard<std::mutex> lk(manifest_mu());
  Manifest m = read_manifest(dir);
  m[name] = r;
  const std::string tmp = dir + "/manifest.json.tmp." + std::to_string(static_cast<long>(getpid()));
  {
    std::ofstream f(tmp);
    if (!f) return;
    f << "{\"format\": 1, \"entries\": {";
    bool first = true;
    for (auto& kv : m) {
      f << (first ? "\n  " : ",\n  ") << '"' << json_escape(kv.first) << "\": {\"hash\": \"" << json_escape(kv.second.hash)
        << "\", \"plan\": \"" << json_escape(kv.second.plan) << "\", \"note\": \"" << json_escape(kv.second.note)
        << "\"}";
      first = false;
    }
    f << "\n}}\n";
  }
  std::rename(tmp.c_str(), (dir + "/manifest.json").c_str());
}

// Tolerance of the first-call check of a fused plan against the generic
// executor: the parity bar itself (1e-5 relative for f32, 2e-2 for bf16,
// per tensor against its largest magnitude), since the generic executor runs
// the module's ops one by one in their own element types, as the reference
// does. SHEAF_B200_VERIFY_RTOL overrides it (tests use it to show that a
// deviation above the bound is rejected).
double verify_tolerance(int dt) {
  const char* e = std::getenv("SHEAF_B200_VERIFY_RTOL");
  if (e && *e) return std::atof(e);
  return dt == DT_BF16 ? 2e-2 : 1e-5;
}

std::string fmt_dev(double v) {
  char b[32];
  std::snprintf(b, sizeof b, "%.2e", v);
  return b;
}

class StableHloModule : public Module {
 public:
  struct Fn {
    std::unique_ptr<GenericFunc> generic;
    std::unique_ptr<Module> fused;  // the fused plan, when recognised and built
    bool vag = false;               // recognised as the nanoGPT value_and_grad (from the text alone)
    bool train = false;             // recognised as the nanoGPT train-step
    bool has_key = false;           // train-step state carries a PRNG key leaf first
    int fused_state = 0;            // 0 = unverified, 1 = verified, -1 = rejected
    int group_state = 0;            // the same, decided jointly by a data-parallel group
    std::string note;
    std::string plan_hash;  // key of the plan cache entry
  };
  std::string cache_dir;
  std::map<std::string, Fn> fns;

  bool has_function(const std::string& fn) const override { return fns.count(fn) != 0; }

  void teardown() override {
    for (auto& kv : fns)
      if (kv.second.fused) kv.second.fused->teardown();
  }

  // Runs the fused plan: value_and_grad as is; train_step without the key
  // leaf (the plan does not use it), which is copied back in front of the
  // new state.
  sb_status fused_call(Session& s, Fn& f, const std::vector<Buffer*>& in, std::vector<Buffer*>& out) {
    if (!f.train) return f.fused->call(s, "value_and_grad", in, out);
    if (!f.has_key) return f.fused->call(s, "train_step", in, out);
    std::vector<Buffer*> rest(in.begin() + 1, in.end());
    std::vector<Buffer*> o;
    SB_TRY(f.fused->call(s, "train_step", rest, o));
    Buffer* key = nullptr;
    sb_status st = buffer_create(s, in[0]->shape, in[0]->elem, &key);
    if (!st && cudaMemcpyAsync(key->data(), in[0]->data(), in[0]->bytes(), cudaMemcpyDeviceToDevice, s.stream) !=
                   cudaSuccess)
      st = make_status(SB_STATUS_INTERNAL, "key copy failed");
    if (st) {
      if (key) buffer_release(key);
      for (Buffer* b : o) buffer_release(b);
      return st;
    }
    out.clear();
    out.push_back(key);
    out.insert(out.end(), o.begin(), o.end());
    return nullptr;
  }

  // This rank's first-call check: the generic executor's outputs (`ref`) and
  // whether the fused plan, run on this rank's inputs alone, agrees with
  // them. Returns an error only when the generic run fails.
  sb_status check_fused(Session& s, Fn& f, const std::vector<Buffer*>& in, std::vector<Buffer*>& ref,
                        std::vector<Buffer*>* keep_fast, bool* agree, std::string* why) {
    *agree = false;
    SB_TRY(f.generic->run(s, in, ref));
    if (!f.fused) {
      *why = "fused plan not built";
      return nullptr;
    }
    std::vector<Buffer*> fast;
    f.fused->set_collectives(false);
    sb_status st = fused_call(s, f, in, fast);
    f.fused->set_collectives(true);
    if (st) {
      *why = sb_status_message(st);
      sb_status_free(st);
      return nullptr;
    }
    double worst = 0;
    sb_status ce = nullptr;
    if (cudaStreamSynchronize(s.stream) != cudaSuccess) {
      ce = make_status(SB_STATUS_INTERNAL, "stream synchronize failed");
    } else if (f.train) {
      const size_t first = f.has_key ? 1 : 0;
      const size_t n = (in.size() - first - 5) / 3;
      std::vector<double> lr;
      ce = host_values(in.back(), &lr);
      if (!ce)
        ce = train_outputs_agree(fast, ref, first, n, lr.empty() ? 0.0 : std::fabs(lr[0]),
                                 verify_tolerance(f.generic->f.args[first].dt), agree, why, &worst);
    } else {
      ce = outputs_agree(fast, ref, verify_tolerance(f.generic->f.args[0].dt), agree, why, &worst);
    }
    if (ce) {
      *agree = false;
      *why = sb_status_message(ce);
      sb_status_free(ce);
    } else {
      *why = (*agree ? "max deviation " : why->empty() ? "max deviation " : *why + "; max deviation ") +
             fmt_dev(worst);
    }
    if (keep_fast && *agree) {
      *keep_fast = fast;
    } else {
      for (Buffer* b : fast) buffer_release(b);
    }
    return nullptr;
  }

  sb_status call(Session& s, const std::string& fn, const std::vector<Buffer*>& in,
                 std::vector<Buffer*>& out) override {
    Fn& f = fns.at(fn);
    if ((f.vag || f.train) && s.comm && s.world > 1) return call_group(s, fn, f, in, out);
    if (f.fused && f.fused_state == 1) return fused_call(s, f, in, out);
    if (f.fused && f.fused_state == 0) {
      std::vector<Buffer*> ref, fast;
      bool agree = false;
      std::string why;
      SB_TRY(check_fused(s, f, in, ref, &fast, &agree, &why));
      if (agree) {
        f.fused_state = 1;
        f.note = std::string(f.train ? "fused nanoGPT train-step plan" : "fused nanoGPT plan") +
                 " (verified against the generic executor on the first call, " + why + ")";
        for (Buffer* b : ref) buffer_release(b);
        out = fast;
      } else {
        f.fused_state = -1;
        f.note = "generic executor (fused plan disagreed: " + why + ")";
        out = ref;
      }
      record_plan(cache_dir, name + "." + fn,
                  PlanRecord{f.plan_hash, f.fused_state == 1 ? "fused-verified" : "fused-rejected", f.note});
      return nullptr;
    }
    return f.generic->run(s, in, out);
  }

  // A recognised value_and_grad in a data-parallel session. Its outputs are
  // the loss and gradients averaged over the group, on either plan: the fused
  // plan all-reduces inside its step, the generic executor's outputs are
  // averaged after it. Which plan runs is decided by all ranks together, so
  // every rank issues the same collectives: on the first call each rank
  // checks the fused plan against the generic executor on its own inputs
  // (plan cache entries are not consulted), then one all-reduce of
  // {agrees, failed} settles it: the fused plan only if every rank agreed,
  // an error on every rank if any rank's generic run failed.
  sb_status call_group(Session& s, const std::string& fn, Fn& f, const std::vector<Buffer*>& in,
                       std::vector<Buffer*>& out) {
    // a train step's outputs are the updated state: they cannot be averaged
    // after the fact, so a group that rejects the fused train plan stops
    const char* no_train = "train_step text in a data-parallel group needs the fused plan, which a rank's first-call "
                           "check rejected";
    if (f.group_state == 1) return fused_call(s, f, in, out);
    if (f.group_state == -1) {
      if (f.train) return make_status(SB_STATUS_UNIMPLEMENTED, no_train);
      SB_TRY(f.generic->run(s, in, out));
      return average_outputs(s, out);
    }
    std::vector<Buffer*> ref;
    bool agree = false;
    std::string why;
    sb_status gen_err = check_fused(s, f, in, ref, nullptr, &agree, &why);
    float flags[2] = {agree ? 1.f : 0.f, gen_err ? 1.f : 0.f};
    Allocation* a = nullptr;
    sb_status xs = session_alloc(s, 256, &a);
    if (!xs) {
      float* d = static_cast<float*>(a->ptr);
      if (cudaMemcpyAsync(d, flags, sizeof flags, cudaMemcpyHostToDevice, s.stream) != cudaSuccess)
        xs = make_status(SB_STATUS_INTERNAL, "flag upload failed");
      if (!xs) xs = comm_allreduce_avg(s, d, 2, SB_ELEM_F32, s.stream);
      if (!xs && (cudaMemcpyAsync(flags, d, sizeof flags, cudaMemcpyDeviceToHost, s.stream) != cudaSuccess ||
                  cudaStreamSynchronize(s.stream) != cudaSuccess))
        xs = make_status(SB_STATUS_INTERNAL, "flag exchange failed");
      allocation_release(a);
    }
    if (xs || gen_err || flags[1] != 0.f) {
      for (Buffer* b : ref) buffer_release(b);
      if (gen_err) {
        if (xs) sb_status_free(xs);
        return gen_err;
      }
      if (xs) return xs;
      return make_status(SB_STATUS_INTERNAL, "the first call failed on another rank of the group");
    }
    // the average of 1/0 flags over the ranks is exactly 1 only if all are 1
    const bool fused = flags[0] == 1.f;
    f.group_state = fused ? 1 : -1;
    f.note = fused ? "fused nanoGPT plan, data-parallel (every rank's first-call check agreed; this rank: " + why + ")"
                   : "generic executor, data-parallel outputs averaged (" +
                         std::string(agree ? "another rank's" : "this rank's") + " first-call check disagreed; " +
                         "this rank: " + why + ")";
    if (s.rank == 0)
      record_plan(cache_dir, name + "." + fn,
                  PlanRecord{f.plan_hash, fused ? "fused-verified" : "fused-rejected", f.note});
    if (fused) {
      for (Buffer* b : ref) buffer_release(b);
      return fused_call(s, f, in, out);
    }
    if (f.train) {
      for (Buffer* b : ref) buffer_release(b);
      return make_status(SB_STATUS_UNIMPLEMENTED, no_train);
    }
    out = ref;
    return average_outputs(s, out);
  }

  // Averages every output over the group (in place, on the session stream).
  static sb_status average_outputs(Session& s, std::vector<Buffer*>& out) {
    for (Buffer* b : out) {
      const size_t es = elem_size(b->elem);
      sb_status st = es ? comm_allreduce_avg(s, b->data(), b->bytes() / es, b->elem, s.stream)
                        : make_status(SB_STATUS_INTERNAL, "output element type");
      if (st) {
        for (Buffer* x : out) buffer_release(x);
        out.clear();
        return st;
      }
    }
    return nullptr;
  }
};

}  // namespace

sb_status load_stablehlo_module(Session& s, const char* text, size_t len, std::unique_ptr<Module>* out) {
  HModule hm;
  try {
    hm = parse_module(text, len);
  } catch (const ParseError& e) {
    return make_status(SB_STATUS_UNIMPLEMENTED, "stablehlo: " + e.msg);
  } catch (const std::exception& e) {
    return make_status(SB_STATUS_INVALID_ARGUMENT, std::string("stablehlo: malformed input (") + e.what() + ")");
  }
  auto m = std::make_unique<StableHloModule>();
  m->name = hm.name;
  m->cache_dir = plan_cache_dir();
  Manifest manifest;
  if (!m->cache_dir.empty()) {
    std::lock_guard<std::mutex> lk(manifest_mu());
    manifest = read_manifest(m->cache_dir);
  }
  const uint64_t text_hash = fnv1a(text, len);
  for (auto& f : hm.funcs) {
    StableHloModule::Fn fn;
    {
      uint64_t h = fnv1a(library_id().data(), library_id().size(), text_hash);
      fn.plan_hash = hex64(fnv1a(f.name.data(), f.name.size(), h));
    }
    const auto rec = manifest.find(hm.name + "." + f.name);
    const bool cached = rec != manifest.end() && rec->second.hash == fn.plan_hash;
    fn.generic = std::make_unique<GenericFunc>();
    fn.generic->f = f;
    try {
      fn.generic->plan();
    } catch (const ParseError& e) {
      return make_status(SB_STATUS_UNIMPLEMENTED, "stablehlo: " + e.msg);
    } catch (const std::exception& e) {
      return make_status(SB_STATUS_INVALID_ARGUMENT, std::string("stablehlo: ") + e.what());
    }
    GptShape g;
    // recognition depends on the text alone, so every rank of a group
    // recognises the same functions whatever its plan cache holds
    fn.vag = match_gpt_vag(fn.generic->f, &g);
    AdamwConfig hp{};
    fn.train = !fn.vag && match_gpt_train(fn.generic->f, &g, &hp, &fn.has_key);
    if (cached && rec->second.plan == "fused-rejected") {
      fn.note = "generic executor (plan cache: " + rec->second.note + ")";
    } else if (fn.vag || fn.train) {
      std::unique_ptr<Module> fused;
      sb_status st = make_gpt_vag_module(s, hm.name + "." + f.name, g, &fused, fn.train ? &hp : nullptr);
      if (!st) {
        fn.fused = std::move(fused);
        const std::string what = fn.train ? "fused nanoGPT train-step plan" : "fused nanoGPT plan";
        if (cached && rec->second.plan == "fused-verified") {
          fn.fused_state = 1;
          fn.note = what + " (verified on an earlier load of this text by this build; plan cache)";
        } else {
          fn.note = what + " pending first-call verification";
        }
      } else {
        fn.note = std::string("generic executor (fused plan unavailable: ") + sb_status_message(st) + ")";
        sb_status_free(st);
      }
    } else {
      fn.note = "generic executor, " + std::to_string(f.ops.size()) + " ops";
    }
    m->fns[f.name] = std::move(fn);
  }
  *out = std::move(m);
  return nullptr;
}

sb_status validate_stablehlo(const char* text, size_t len, std::string* summary) {
  try {
    HModule hm = parse_module(text, len);
    std::ostringstream os;
    os << "module @" << hm.name;
    for (auto& f : hm.funcs) {
      GenericFunc g;
      g.f = f;
      g.plan();
      GptShape gs;
      os << "\n" << f.name << ": " << f.ops.size() << " ops, " << f.args.size() << " args, " << f.rets.size()
         << " results, arena " << g.arena_bytes << " B";
      AdamwConfig hp{};
      bool key = false;
      if (match_gpt_vag(g.f, &gs))
        os << ", nanoGPT value_and_grad L=" << gs.n_layer << " H=" << gs.n_head << " D=" << gs.n_embd
           << " V=" << gs.vocab << " B=" << gs.batch << " T=" << gs.seq;
      else if (match_gpt_train(g.f, &gs, &hp, &key))
        os << ", nanoGPT train_step L=" << gs.n_layer << " H=" << gs.n_head << " D=" << gs.n_embd
           << " V=" << gs.vocab << " B=" << gs.batch << " T=" << gs.seq << " b1=" << hp.b1 << " b2=" << hp.b2
           << " eps=" << hp.eps << " wd=" << hp.wd << " max_norm=" << hp.max_norm << (key ? " (key leaf)" : "");
    }
    if (summary) *summary = os.str();
  } catch (const ParseError& e) {
    return make_status(SB_STATUS_UNIMPLEMENTED, "stablehlo: " + e.msg);
  } catch (const std::exception& e) {
    return make_status(SB_STATUS_INVALID_ARGUMENT, std::string("stablehlo: ") + e.what());
  }
  return nullptr;
}

std::string describe_stablehlo_module(Module* mod) {
  auto* m = dynamic_cast<StableHloModule*>(mod);
  if (!m) return "fused module (created from a configuration)";
  std::ostringstream os;
  for (auto& kv : m->fns) os << kv.first << ": " << kv.second.note << "\n";
  return os.str();
}

}  // namespace sb

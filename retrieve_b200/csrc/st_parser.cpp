// SilverTorch's expression-query parser on the host: the query DSL
//
//   expression := or_expr
//   or_expr    := and_expr (("OR" | "|") and_expr)*
//   and_expr   := unary (("AND" | "&") unary)*
//   unary      := ("NOT" | "!") unary | primary
//   primary    := "(" expression ")" | id ":" value [":" weight]
//
// (silvertorch/ops/csrc/EXPRESSION_SYNTAX.md) compiled to the postfix bloom plans that
// st::search, the bloom searches and rb_st_bloom_* evaluate, in the parser's byte encoding
// (st::parse_expression_query_batch, expression_query_parser.cpp:395-430; encoding
// bloom_index_util.cpp:27-127), so the plans are byte-identical to the reference's:
//
//  * operators: AND 1, OR 2, NOT 3, TERM 4, EMPTY 5 (one byte each); a compound operator's
//    parameters are the indices of its children's root operators, a term's its term number;
//  * an AND / OR chain becomes one operator over all its operands, except that every time
//    max_sub_queries operands have gathered they are folded into one operator, which becomes
//    the first operand of the rest (and a chain that folded gets its closing operator even
//    over a single operand); a chain of one operand adds no operator;
//  * a term carries bloom_hash_k stored hashes MurmurHash3(id, value, seed) for seeds
//    0 .. bloom_hash_k - 1; the weight is parsed and dropped; the empty expression is the
//    match-all plan [EMPTY];
//  * per plan, four segments appended to the data, each padded to 8 bytes: operators (u8),
//    the running parameter counts (i32, a leading 0, one entry per operator), parameters
//    (i32), hashes (u64); eight offsets per plan give each segment's [start, end) bytes.
//
// The tokens and plans are built here in a structure of this file's own; what must match the
// reference is the accepted language, the emission order and the encoding above.
#include <cctype>
#include <cerrno>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "bloom_hash.cuh"
#include "retrieve_b200.h"

namespace rb {
void set_last_error(const char* msg);

namespace {

enum : uint8_t { kOpAnd = 1, kOpOr = 2, kOpNot = 3, kOpTerm = 4, kOpEmpty = 5 };
enum class Tok { Int, Real, Colon, LParen, RParen, And, Or, Not, End };
constexpr int kMaxDepth = 1024;  // recursion depth accepted: 3 levels a parenthesis, 1 a NOT

struct Token {
  Tok kind;
  size_t pos, len;
};

struct ParseError {
  std::string msg;
};

[[noreturn]] void fail(const std::string& what, size_t pos) {
  throw ParseError{what + " at position " + std::to_string(pos)};
}

// The whole expression as tokens, END last. A number is an optional '-' directly followed
// by digits, then digits and at most one '.'; a word is a run of letters.
std::vector<Token> tokenize(const char* s, size_t n) {
  std::vector<Token> out;
  size_t i = 0;
  while (true) {
    while (i < n && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
    if (i >= n) break;
    const size_t start = i;
    const char c = s[i];
    Tok kind;
    if (c == '(' || c == ')' || c == ':' || c == '&' || c == '|' || c == '!') {
      kind = c == '(' ? Tok::LParen : c == ')' ? Tok::RParen : c == ':' ? Tok::Colon
           : c == '&' ? Tok::And : c == '|' ? Tok::Or : Tok::Not;
      ++i;
    } else if (std::isdigit(static_cast<unsigned char>(c)) ||
               (c == '-' && i + 1 < n && std::isdigit(static_cast<unsigned char>(s[i + 1])))) {
      bool dot = false;
      if (c == '-') ++i;
      while (i < n && (std::isdigit(static_cast<unsigned char>(s[i])) || s[i] == '.')) {
        if (s[i] == '.') {
          if (dot) break;
          dot = true;
        }
        ++i;
      }
      kind = dot ? Tok::Real : Tok::Int;
    } else if (std::isalpha(static_cast<unsigned char>(c))) {
      while (i < n && std::isalpha(static_cast<unsigned char>(s[i]))) ++i;
      const std::string word(s + start, i - start);
      if (word == "AND") kind = Tok::And;
      else if (word == "OR") kind = Tok::Or;
      else if (word == "NOT") kind = Tok::Not;
      else fail("unknown keyword '" + word + "'", start);
    } else {
      fail(std::string("unexpected character '") + c + "'", start);
    }
    out.push_back({kind, start, i - start});
  }
  out.push_back({Tok::End, n, 0});
  return out;
}

struct Plan {
  std::vector<uint8_t> ops;
  std::vector<int32_t> param_end{0};  // running parameter count, one more entry than ops
  std::vector<int32_t> params;
  std::vector<uint64_t> hashes;
};

class PlanBuilder {
 public:
  PlanBuilder(const char* s, size_t n, Plan& plan, int64_t hash_k, int64_t max_sub)
      : src_(s), toks_(tokenize(s, n)), plan_(plan), hash_k_(hash_k), max_sub_(max_sub) {}

  void run() {
    chain(Tok::Or, kOpOr, 0);
    if (peek().kind != Tok::End) fail("unexpected token '" + text(peek()) + "', expected the end", peek().pos);
  }

 private:
  const Token& peek() const { return toks_[at_]; }
  Token take() { return toks_[at_ < toks_.size() - 1 ? at_++ : at_]; }
  std::string text(const Token& t) const { return std::string(src_ + t.pos, t.len); }
  int32_t root() const { return static_cast<int32_t>(plan_.ops.size()) - 1; }

  void emit(uint8_t op, const std::vector<int32_t>& children) {
    plan_.params.insert(plan_.params.end(), children.begin(), children.end());
    plan_.ops.push_back(op);
    plan_.param_end.push_back(plan_.param_end.back() + static_cast<int32_t>(children.size()));
  }

  // One precedence level: operands joined by `sep` into `op` operators (OR over AND chains,
  // AND over unary operands), folded every max_sub_queries operands.
  void chain(Tok sep, uint8_t op, int depth) {
    if (depth > kMaxDepth) fail("expression nested too deeply", peek().pos);
    std::vector<int32_t> operands;
    bool folded = false;
    auto operand = [&] {
      if (sep == Tok::Or) chain(Tok::And, kOpAnd, depth + 1);
      else unary(depth + 1);
      operands.push_back(root());
    };
    auto fold = [&] {
      if (static_cast<int64_t>(operands.size()) == max_sub_) {
        emit(op, operands);
        operands.assign(1, root());
        folded = true;
      }
    };
    operand();
    if (peek().kind == sep) fold();
    while (peek().kind == sep) {
      take();
      operand();
      fold();
    }
    if (operands.size() > 1 || folded) emit(op, operands);
  }

  void unary(int depth) {
    if (depth > kMaxDepth) fail("expression nested too deeply", peek().pos);
    if (peek().kind == Tok::Not) {
      take();
      unary(depth + 1);
      emit(kOpNot, {root()});
      return;
    }
    if (peek().kind == Tok::LParen) {
      take();
      chain(Tok::Or, kOpOr, depth + 1);
      const Token close = take();
      if (close.kind != Tok::RParen) fail("expected ')', got '" + text(close) + "'", close.pos);
      return;
    }
    term();
  }

  int64_t integer(const char* what) {
    const Token t = take();
    if (t.kind != Tok::Int) fail(std::string("expected ") + what + " (integer), got '" + text(t) + "'", t.pos);
    const std::string s = text(t);
    errno = 0;
    char* end = nullptr;
    const long long v = std::strtoll(s.c_str(), &end, 10);
    if (errno == ERANGE || end != s.c_str() + s.size()) fail(std::string(what) + " '" + s + "' out of range", t.pos);
    return static_cast<int64_t>(v);
  }

  void term() {
    const int64_t id = integer("feature id");
    const Token colon = take();
    if (colon.kind != Tok::Colon) fail("expected ':' after the feature id", colon.pos);
    const int64_t value = integer("feature value");
    if (peek().kind == Tok::Colon) {  // id:value:weight, the weight is not part of the plan
      take();
      const Token w = take();
      if (w.kind != Tok::Int && w.kind != Tok::Real) fail("expected a weight, got '" + text(w) + "'", w.pos);
    }
    for (int64_t seed = 0; seed < hash_k_; ++seed)
      plan_.hashes.push_back(murmur3_pair(static_cast<uint64_t>(id), static_cast<uint64_t>(value),
                                          static_cast<uint64_t>(seed)));
    plan_.ops.push_back(kOpTerm);
    plan_.param_end.push_back(plan_.param_end.back() + 1);
    plan_.params.push_back(static_cast<int32_t>(plan_.hashes.size() / hash_k_) - 1);
  }

  const char* src_;
  std::vector<Token> toks_;
  size_t at_ = 0;
  Plan& plan_;
  int64_t hash_k_, max_sub_;
};

// Deepest operand stack of the plan's postfix evaluation (a compound operator pops its
// children and pushes its result).
int64_t stack_depth(const Plan& p) {
  int64_t depth = 0, sp = 0;
  for (size_t j = 0; j < p.ops.size(); ++j) {
    if (p.ops[j] == kOpTerm || p.ops[j] == kOpEmpty) sp += 1;
    else sp += 1 - (p.param_end[j + 1] - p.param_end[j]);
    if (sp > depth) depth = sp;
  }
  return depth;
}

template <typename T>
void append_segment(const std::vector<T>& v, std::vector<uint8_t>& data, int64_t* offsets) {
  const size_t start = data.size(), bytes = v.size() * sizeof(T);
  data.resize(start + (bytes + 7) / 8 * 8, 0);
  if (bytes) std::memcpy(data.data() + start, v.data(), bytes);
  offsets[0] = static_cast<int64_t>(start);
  offsets[1] = static_cast<int64_t>(start + bytes);
}

}  // namespace
}  // namespace rb

extern "C" {

int rb_st_parse_expression_batch(const char* const* expressions, const int64_t* lengths, int n_expressions,
                                 int64_t bloom_hash_k, int64_t max_sub_queries, int8_t* out_data,
                                 int64_t data_capacity, int64_t* out_offsets, int64_t* out_data_bytes,
                                 int64_t* out_max_stack) {
  using namespace rb;
  if (n_expressions < 0 || (n_expressions > 0 && (expressions == nullptr || lengths == nullptr)) ||
      out_data_bytes == nullptr || out_max_stack == nullptr || bloom_hash_k < 1 || bloom_hash_k > (1 << 20)) {
    set_last_error("parse_expression_query_batch: bad arguments (bloom_hash_k must be in [1, 2^20])");
    return RB_ERR_INVALID_ARG;
  }
  std::vector<uint8_t> data;
  std::vector<int64_t> offsets(8 * static_cast<size_t>(n_expressions));
  int64_t depth = 0;
  try {
    for (int e = 0; e < n_expressions; ++e) {
      if (lengths[e] < 0 || (lengths[e] > 0 && expressions[e] == nullptr)) {
        set_last_error("parse_expression_query_batch: bad expression length");
        return RB_ERR_INVALID_ARG;
      }
      Plan plan;
      if (lengths[e] == 0) {
        plan.ops.push_back(kOpEmpty);  // the empty expression matches every doc
        plan.param_end.push_back(0);
      } else {
        PlanBuilder(expressions[e], static_cast<size_t>(lengths[e]), plan, bloom_hash_k, max_sub_queries).run();
      }
      const int64_t d = stack_depth(plan);
      if (d > depth) depth = d;
      int64_t* o = offsets.data() + 8 * static_cast<size_t>(e);
      append_segment(plan.ops, data, o);
      append_segment(plan.param_end, data, o + 2);
      append_segment(plan.params, data, o + 4);
      append_segment(plan.hashes, data, o + 6);
    }
  } catch (const ParseError& err) {
    set_last_error(("parse_expression_query_batch: " + err.msg).c_str());
    return RB_ERR_INVALID_ARG;
  } catch (const std::exception& err) {
    set_last_error(err.what());
    return RB_ERR_INVALID_ARG;
  }
  *out_data_bytes = static_cast<int64_t>(data.size());
  *out_max_stack = depth;
  if (out_data == nullptr && out_offsets == nullptr) return RB_OK;  // size query
  if (out_offsets == nullptr || (!data.empty() && (out_data == nullptr || data_capacity < *out_data_bytes))) {
    set_last_error("parse_expression_query_batch: output buffers too small");
    return RB_ERR_WORKSPACE;
  }
  if (!data.empty()) std::memcpy(out_data, data.data(), data.size());
  if (!offsets.empty()) std::memcpy(out_offsets, offsets.data(), offsets.size() * sizeof(int64_t));
  return RB_OK;
}

}  // extern "C"

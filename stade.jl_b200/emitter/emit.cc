// emit.cc -- the .cu emitter (include/stade_emit.h).
//
// Input: the Julia subset STADE's generators write (agen_emit, tgen_emit,
// hvp_emit): functions of `for v = lo[:step]:hi`, `if / elseif / else`,
// `while`, assignments to scalars and to array elements `a[i]`, `a[i, j]`,
// integer index arithmetic (div / mod / max / min), float arithmetic with the
// der_ table's functions, `return nothing | x | (x, y, ...)`; and the
// initstacks function (`s = Vector{Float64}(undef, n)`, `return (s, ...)`).
//
// Output: CUDA C++ for sm_100a. The decisions follow cgen_body
// (src/STADE.jl:10409-10640) in spirit, by this module's own rules:
//   - a loop becomes a kernel with one thread per iteration when no value
//     flows between iterations: every scalar it assigns is private to an
//     iteration (first referenced by an unconditional write, not read after
//     the loop before being rewritten; or reset to the same literal at the end
//     of every iteration and holding it on entry, the convergent constant of
//     cgen_split_loop_gate) or is only accumulated (`s = s + e`, an atomic add
//     into the scalar's device box, as cgen_device_assign boxes reduction
//     scalars); every array it writes is either written and read at one
//     injective index of the thread variable (plain stores) or only
//     accumulated into (atomic adds, as cgen_device_assign's atomics);
//   - a loop that does not qualify but holds loops that do stays a host loop
//     (its variable passed to the kernels by value), as cgen_body recurses;
//   - everything else (scalar statements, `while`, loops carrying a value)
//     runs in order in a one-thread kernel, keeping device state on the
//     device (the generated CUDA.jl code runs those on the host under
//     allowscalar).
// Scalars live in registers when one kernel uses them, else in a device box
// (`g_fbox` / `g_ibox`); integer scalars computed on the host from the integer
// arguments, and float arguments the sweep never assigns, are kernel
// arguments. A parallel loop holding block sums strides over its iterations
// with the grid the device holds at once. No host synchronisation happens before the
// end, where returned scalar adjoints are copied back.
//
// Index injectivity: an index is injective in the thread variable v when one
// of its dimensions is a v * a + b with a, b loop-invariant, or two dimensions
// are div(X, n) and mod(X, n) of the same injective X (the flattened-nest
// decode of skill-stade rule 4), or one dimension is
// (div(X, n) + c) * n + mod(X, n) + c' (the re-flattened index).
#include "stade_emit.h"

#include <algorithm>
#include <cctype>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <sstream>
#include <stdexcept>
#include <string>
#include <vector>

namespace stade_emit {

struct Error : std::runtime_error {
  using std::runtime_error::runtime_error;
};

[[noreturn]] void fail(int line, const std::string& msg) {
  throw Error(line > 0 ? "line " + std::to_string(line) + ": " + msg : msg);
}

// ---- lexer -------------------------------------------------------------------
enum TokKind { T_NAME, T_NUM, T_OP, T_NL, T_EOF };
struct Tok {
  TokKind k;
  std::string s;
  int line;
};

std::vector<Tok> lex(const std::string& src) {
  std::vector<Tok> out;
  int line = 1;
  size_t i = 0, n = src.size();
  auto push = [&](TokKind k, std::string s) {
    if (k == T_NL && (out.empty() || out.back().k == T_NL)) return;
    out.push_back({k, std::move(s), line});
  };
  while (i < n) {
    const char c = src[i];
    if (c == '#') {
      while (i < n && src[i] != '\n') ++i;
      continue;
    }
    if (c == '\n' || c == ';') {
      push(T_NL, "\n");
      if (c == '\n') ++line;
      ++i;
      continue;
    }
    if (c == ' ' || c == '\t' || c == '\r') {
      ++i;
      continue;
    }
    if (std::isalpha((unsigned char)c) || c == '_' || c == '@') {
      size_t j = i + 1;
      while (j < n && (std::isalnum((unsigned char)src[j]) || src[j] == '_' || src[j] == '!')) ++j;
      push(T_NAME, src.substr(i, j - i));
      i = j;
      continue;
    }
    if (std::isdigit((unsigned char)c) ||
        (c == '.' && i + 1 < n && std::isdigit((unsigned char)src[i + 1]))) {
      size_t j = i;
      bool flt = false;
      while (j < n && std::isdigit((unsigned char)src[j])) ++j;
      if (j < n && src[j] == '.' && !(j + 1 < n && src[j + 1] == '.')) {
        flt = true;
        ++j;
        while (j < n && std::isdigit((unsigned char)src[j])) ++j;
      }
      if (j < n && (src[j] == 'e' || src[j] == 'E' || src[j] == 'f') &&
          j + 1 < n && (std::isdigit((unsigned char)src[j + 1]) ||
                        ((src[j + 1] == '-' || src[j + 1] == '+') && j + 2 < n &&
                         std::isdigit((unsigned char)src[j + 2])))) {
        flt = true;
        j += 2;
        while (j < n && std::isdigit((unsigned char)src[j])) ++j;
      }
      std::string t = src.substr(i, j - i);
      for (auto& ch : t)
        if (ch == 'f') ch = 'e';   // 1.0f0 (Float32 literal) -> 1.0e0
      push(T_NUM, flt ? t + (t.find('.') == std::string::npos && t.find('e') == std::string::npos
                                 ? ".0" : "")
                      : t);
      i = j;
      // a numeric literal coefficient (`0.5__oldb_0`, `2(x + 1)`): multiplication
      if (i < n && (std::isalpha((unsigned char)src[i]) || src[i] == '_' || src[i] == '('))
        push(T_OP, "jux");
      continue;
    }
    static const char* two[] = {"==", "!=", "<=", ">=", "&&", "||", "+=", "-=", "*=", "/="};
    bool matched = false;
    for (const char* op : two)
      if (src.compare(i, 2, op) == 0) {
        push(T_OP, op);
        i += 2;
        matched = true;
        break;
      }
    if (matched) continue;
    if (std::strchr("+-*/^()[],=<>!:{}%", c)) {
      push(T_OP, std::string(1, c));
      ++i;
      continue;
    }
    if ((unsigned char)c == 0xC3 && i + 1 < n && (unsigned char)src[i + 1] == 0xB7) {  // ÷
      push(T_OP, "÷");
      i += 2;
      continue;
    }
    fail(line, std::string("unexpected character '") + c + "'");
  }
  push(T_NL, "\n");
  out.push_back({T_EOF, "", line});
  return out;
}

// ---- AST ---------------------------------------------------------------------
struct Expr;
using EP = std::shared_ptr<Expr>;
struct Expr {
  enum Kind { Num, Var, Ref, Call, Bin, Un, Tuple, Curly } kind;
  std::string s;       // number text, name, array, function, operator
  bool int_lit = false;
  std::vector<EP> a;   // operands, indices, arguments
};

struct Stmt;
using SP = std::shared_ptr<Stmt>;
struct Stmt {
  enum Kind { Assign, For, If, While, Return } kind;
  int line = 0;
  EP lhs, rhs;                  // Assign
  std::string var;              // For
  EP lo, step, hi;              // For (step null = 1)
  EP cond;                      // If, While
  std::vector<SP> body, els;    // For / While / If-then, If-else
  EP ret;                       // Return (null: nothing)
  // parent links, filled after parsing
  std::vector<SP>* in = nullptr;
  size_t pos = 0;
  Stmt* owner = nullptr;        // enclosing For / While / If (null: function body)
};

struct Func {
  std::string name;
  std::vector<std::string> params;
  std::vector<SP> body;
  int line = 0;
};

EP mk(Expr::Kind k, std::string s, std::vector<EP> a = {}) {
  auto e = std::make_shared<Expr>();
  e->kind = k;
  e->s = std::move(s);
  e->a = std::move(a);
  return e;
}

// ---- parser ------------------------------------------------------------------
class Parser {
 public:
  explicit Parser(std::vector<Tok> t) : t_(std::move(t)) {}

  std::vector<Func> file() {
    std::vector<Func> fs;
    skip_nl();
    while (peek().k != T_EOF) {
      if (is_name("function")) {
        fs.push_back(function());
      } else {
        // anything else at top level (using, comments' leftovers): skip a line
        while (peek().k != T_NL && peek().k != T_EOF) next();
      }
      skip_nl();
    }
    return fs;
  }

 private:
  std::vector<Tok> t_;
  size_t p_ = 0;

  const Tok& peek(size_t o = 0) const { return t_[std::min(p_ + o, t_.size() - 1)]; }
  Tok next() { return t_[p_ < t_.size() - 1 ? p_++ : p_]; }
  bool is_op(const char* s, size_t o = 0) const { return peek(o).k == T_OP && peek(o).s == s; }
  bool is_name(const char* s) const { return peek().k == T_NAME && peek().s == s; }
  void expect_op(const char* s) {
    if (!is_op(s)) fail(peek().line, std::string("expected '") + s + "', found '" + peek().s + "'");
    next();
  }
  std::string expect_name() {
    if (peek().k != T_NAME) fail(peek().line, "expected a name, found '" + peek().s + "'");
    return next().s;
  }
  void skip_nl() {
    while (peek().k == T_NL) next();
  }
  void end_stmt() {
    if (peek().k != T_NL && peek().k != T_EOF && !is_name("end"))
      fail(peek().line, "unexpected '" + peek().s + "' after a statement");
    skip_nl();
  }

  Func function() {
    Func f;
    f.line = peek().line;
    next();  // function
    f.name = expect_name();
    expect_op("(");
    while (!is_op(")")) {
      f.params.push_back(expect_name());
      if (is_op(",")) next();
      else if (!is_op(")")) fail(peek().line, "expected ',' or ')' in the parameter list");
    }
    next();
    skip_nl();
    f.body = block({"end"});
    next();  // end
    return f;
  }

  std::vector<SP> block(std::initializer_list<const char*> stops) {
    std::vector<SP> out;
    for (;;) {
      skip_nl();
      if (peek().k == T_EOF) fail(peek().line, "missing 'end'");
      for (const char* s : stops)
        if (is_name(s)) return out;
      out.push_back(statement());
    }
  }

  SP statement() {
    auto st = std::make_shared<Stmt>();
    st->line = peek().line;
    if (peek().k == T_NAME && peek().s[0] == '@') {  // @inbounds and the like: ignored
      next();
      return statement();
    }
    if (is_name("local")) {
      next();
      // `local x` / `local x = e`
      if (peek().k == T_NAME && (peek(1).k == T_NL || peek(1).k == T_EOF)) {
        next();
        skip_nl();
        return statement();
      }
    }
    if (is_name("for")) {
      next();
      st->kind = Stmt::For;
      st->var = expect_name();
      if (is_op("=")) next();
      else if (is_name("in")) next();
      else fail(peek().line, "expected '=' or 'in' after the loop variable");
      EP a = arith();
      expect_op(":");
      EP b = arith();
      if (is_op(":")) {
        next();
        st->lo = a;
        st->step = b;
        st->hi = arith();
      } else {
        st->lo = a;
        st->hi = b;
      }
      skip_nl();
      st->body = block({"end"});
      next();
      end_stmt();
      return st;
    }
    if (is_name("while")) {
      next();
      st->kind = Stmt::While;
      st->cond = expr();
      skip_nl();
      st->body = block({"end"});
      next();
      end_stmt();
      return st;
    }
    if (is_name("if")) {
      next();
      if_tail(st);
      end_stmt();
      return st;
    }
    if (is_name("return")) {
      next();
      st->kind = Stmt::Return;
      if (peek().k != T_NL && !is_name("end")) {
        if (is_name("nothing")) {
          next();
        } else {
          EP e = expr();
          if (is_op(",")) {
            std::vector<EP> items{e};
            while (is_op(",")) {
              next();
              items.push_back(expr());
            }
            e = mk(Expr::Tuple, "", items);
          }
          st->ret = e;
        }
      }
      end_stmt();
      return st;
    }
    // assignment
    EP lhs = postfix();
    if (lhs->kind != Expr::Var && lhs->kind != Expr::Ref)
      fail(st->line, "left-hand side must be a variable or an array element");
    st->kind = Stmt::Assign;
    st->lhs = lhs;
    if (is_op("=")) {
      next();
      st->rhs = expr();
    } else if (is_op("+=") || is_op("-=") || is_op("*=") || is_op("/=")) {
      std::string op = next().s.substr(0, 1);
      st->rhs = mk(Expr::Bin, op, {lhs, expr()});
    } else {
      fail(st->line, "expected '=' in an assignment, found '" + peek().s + "'");
    }
    end_stmt();
    return st;
  }

  // after `if` / `elseif`: cond, then-block, and the rest; consumes the final `end`
  void if_tail(SP& st) {
    st->kind = Stmt::If;
    st->cond = expr();
    skip_nl();
    st->body = block({"elseif", "else", "end"});
    if (is_name("elseif")) {
      next();
      auto sub = std::make_shared<Stmt>();
      sub->line = peek().line;
      if_tail(sub);
      st->els.push_back(sub);
      return;
    }
    if (is_name("else")) {
      next();
      skip_nl();
      st->els = block({"end"});
    }
    next();  // end
  }

  EP expr() { return lor(); }
  EP lor() {
    EP l = land();
    while (is_op("||")) {
      next();
      l = mk(Expr::Bin, "||", {l, land()});
    }
    return l;
  }
  EP land() {
    EP l = cmp();
    while (is_op("&&")) {
      next();
      l = mk(Expr::Bin, "&&", {l, cmp()});
    }
    return l;
  }
  EP cmp() {
    EP l = arith();
    for (const char* op : {"==", "!=", "<=", ">=", "<", ">"})
      if (is_op(op)) {
        next();
        EP r = arith();
        for (const char* op2 : {"==", "!=", "<=", ">=", "<", ">"})
          if (is_op(op2)) fail(peek().line, "chained comparisons are not supported");
        return mk(Expr::Bin, op, {l, r});
      }
    return l;
  }
  EP arith() {
    EP l = term();
    while (is_op("+") || is_op("-")) {
      std::string op = next().s;
      l = mk(Expr::Bin, op, {l, term()});
    }
    return l;
  }
  EP term() {
    EP l = unary();
    while (is_op("*") || is_op("/") || is_op("%") || is_op("÷")) {
      std::string op = next().s;
      l = mk(Expr::Bin, op, {l, unary()});
    }
    return l;
  }
  EP unary() {
    if (is_op("-") || is_op("+") || is_op("!")) {
      std::string op = next().s;
      EP e = unary();
      if (op == "+") return e;
      if (op == "-" && e->kind == Expr::Num && e->s[0] != '-') {
        EP n = mk(Expr::Num, "-" + e->s);
        n->int_lit = e->int_lit;
        return n;
      }
      return mk(Expr::Un, op, {e});
    }
    return power();
  }
  EP power() {
    EP b = postfix();
    if (b->kind == Expr::Num && is_op("jux")) {
      // Julia: a literal coefficient binds tighter than * and / (1/2x is
      // 1/(2x)) and takes the power after it (2x^3 is 2(x^3))
      next();
      return mk(Expr::Bin, "*", {b, power()});
    }
    if (is_op("^")) {
      next();
      return mk(Expr::Bin, "^", {b, unary()});
    }
    return b;
  }
  EP postfix() {
    EP e = primary();
    for (;;) {
      if (is_op("[") && e->kind == Expr::Var) {
        next();
        std::vector<EP> idx;
        while (!is_op("]")) {
          idx.push_back(expr());
          if (is_op(",")) next();
          else if (!is_op("]")) fail(peek().line, "expected ',' or ']' in an index");
        }
        next();
        e = mk(Expr::Ref, e->s, idx);
      } else if (is_op("(") && (e->kind == Expr::Var || e->kind == Expr::Curly)) {
        next();
        std::vector<EP> args;
        while (!is_op(")")) {
          args.push_back(expr());
          if (is_op(",")) next();
          else if (!is_op(")")) fail(peek().line, "expected ',' or ')' in a call");
        }
        next();
        if (e->kind == Expr::Curly) {
          e->a = args;   // Vector{T}(undef, n): type in s, arguments in a
        } else {
          e = mk(Expr::Call, e->s, args);
        }
      } else if (is_op("{") && e->kind == Expr::Var) {
        next();
        std::string inner = expect_name();
        expect_op("}");
        e = mk(Expr::Curly, e->s + "{" + inner + "}");
      } else {
        return e;
      }
    }
  }
  EP primary() {
    const Tok& t = peek();
    if (t.k == T_NUM) {
      next();
      EP e = mk(Expr::Num, t.s);
      e->int_lit = t.s.find_first_of(".eE") == std::string::npos;
      return e;
    }
    if (t.k == T_NAME) {
      next();
      if (t.s == "true" || t.s == "false") {
        EP e = mk(Expr::Num, t.s == "true" ? "1" : "0");
        e->int_lit = true;
        return e;
      }
      return mk(Expr::Var, t.s);
    }
    if (is_op("(")) {
      next();
      EP e = expr();
      if (is_op(",")) {
        std::vector<EP> items{e};
        while (is_op(",")) {
          next();
          if (is_op(")")) break;
          items.push_back(expr());
        }
        expect_op(")");
        return mk(Expr::Tuple, "", items);
      }
      expect_op(")");
      return e;
    }
    fail(t.line, "unexpected '" + t.s + "' in an expression");
  }
};

void link(std::vector<SP>& body, Stmt* owner) {
  for (size_t i = 0; i < body.size(); ++i) {
    Stmt* s = body[i].get();
    s->in = &body;
    s->pos = i;
    s->owner = owner;
    link(s->body, s);
    link(s->els, s);
  }
}

// ---- expression helpers ------------------------------------------------------
std::string text(const EP& e) {
  switch (e->kind) {
    case Expr::Num:
    case Expr::Var:
      return e->s;
    case Expr::Ref:
    case Expr::Call: {
      std::string s = e->s + (e->kind == Expr::Ref ? "[" : "(");
      for (size_t i = 0; i < e->a.size(); ++i) s += (i ? ", " : "") + text(e->a[i]);
      return s + (e->kind == Expr::Ref ? "]" : ")");
    }
    case Expr::Bin:
      return "(" + text(e->a[0]) + " " + e->s + " " + text(e->a[1]) + ")";
    case Expr::Un:
      return e->s + text(e->a[0]);
    case Expr::Tuple: {
      std::string s = "(";
      for (size_t i = 0; i < e->a.size(); ++i) s += (i ? ", " : "") + text(e->a[i]);
      return s + ")";
    }
    case Expr::Curly:
      return e->s;
  }
  return "?";
}

void walk_expr(const EP& e, const std::function<void(const EP&)>& f) {
  if (!e) return;
  f(e);
  for (auto& c : e->a) walk_expr(c, f);
}

void walk_stmts(const std::vector<SP>& b, const std::function<void(Stmt&)>& f) {
  for (auto& s : b) {
    f(*s);
    walk_stmts(s->body, f);
    walk_stmts(s->els, f);
  }
}

// scalar names read by an expression (array names excluded)
void scalar_reads(const EP& e, std::set<std::string>& out) {
  walk_expr(e, [&](const EP& x) {
    if (x->kind == Expr::Var) out.insert(x->s);
  });
}
bool reads_scalar(const EP& e, const std::string& v) {
  std::set<std::string> r;
  scalar_reads(e, r);
  return r.count(v) > 0;
}
bool reads_array(const EP& e, const std::string& a) {
  bool hit = false;
  walk_expr(e, [&](const EP& x) {
    if (x->kind == Expr::Ref && x->s == a) hit = true;
  });
  return hit;
}

// ---- the emitter -------------------------------------------------------------
struct LoopPlan {
  bool parallel = false;
  std::string why;
  std::map<std::string, std::string> privates;   // name -> initial literal ("" none)
  std::set<std::string> reductions;
  std::set<std::string> atomic_arrays;
};

enum Storage { S_HOSTINT, S_LOCAL, S_FBOX, S_IBOX, S_FPARAM };

// The iteration v whose accumulation lands on target index j, for one
// accumulation statement (the scatter -> gather rewrite, as cgen_gather_loop
// and cgen_gather_periodic_inverse, src/STADE.jl:7343-7532).
struct Inverse {
  enum Kind { IDENT, OFFSET, PERIODIC2 } kind = IDENT;
  long off = 0;        // OFFSET: the index is v + off
  EP n;                // PERIODIC2: v = (i - 1) n + j decoded on an n x n grid
  long sr = 0, sc = 0; // PERIODIC2: periodic row / column shift of the target
};
struct GatherPart {
  Stmt* st;
  EP term;
  Inverse inv;
};
struct Gather {
  std::string array;
  std::vector<GatherPart> parts;
};

struct Unit {
  bool par = false;
  bool gather = false;        // a gather kernel (stmts = {the original loop})
  std::vector<Gather> gathers;
  std::vector<SP> stmts;      // SEQ: statements in order; PAR: the one For
  LoopPlan plan;
  std::set<std::string> scalars, arrays;  // referenced
  std::set<std::string> inner_vars;       // loop variables of loops inside
  int id = 0;
};

struct Item {
  enum Kind { HostAssign, HostFor, HostIf, Kernel, Return } kind;
  SP st;
  std::vector<Item> a, b;
  int unit = -1;
};

struct Cls {
  enum K { INV, INJ, DIVP, MODP, MULDIV, OTHER } k = OTHER;
  std::string key, n;
};

class Emitter {
 public:
  Emitter(Func& f, const Func* init, int precision, const std::string& dims_spec)
      : f_(f), init_(init), f32_(precision == 32) {
    T_ = f32_ ? "float" : "double";
    link(f_.body, nullptr);
    scope_loop_vars();
    hoist_local_arrays();
    for (auto& p : f_.params) params_.insert(p);
    parse_dims(dims_spec);
    infer_kinds();
  }

  std::string cu, manifest;

  // A Julia loop variable is local to its loop. Where a loop's variable name
  // is also assigned outside that loop (transformer_b: `for i = 1:n` as a host
  // loop, `i = div(...)` in a later kernel), the loop's own `i` is renamed
  // `i__<line>` in its header and body, so that one name is one variable.
  void scope_loop_vars() {
    std::vector<Stmt*> loops;
    walk_stmts(f_.body, [&](Stmt& x) {
      if (x.kind == Stmt::For) loops.push_back(&x);
    });
    for (Stmt* F : loops) {
      const std::string v = F->var;
      bool outside = false;
      walk_stmts(f_.body, [&](Stmt& x) {
        if (x.kind != Stmt::Assign || x.lhs->kind != Expr::Var || x.lhs->s != v) return;
        bool inside = false;
        for (Stmt* o = x.owner; o; o = o->owner) inside = inside || o == F;
        if (!inside) outside = true;
      });
      if (!outside) continue;
      const std::string w = v + "__" + std::to_string(F->line);
      F->var = w;
      rename_in(F->body, v, w);
    }
  }
  static void rename_expr(const EP& e, const std::string& v, const std::string& w) {
    if (!e) return;
    walk_expr(e, [&](const EP& x) {
      if (x->kind == Expr::Var && x->s == v) x->s = w;
    });
  }
  static void rename_in(std::vector<SP>& body, const std::string& v, const std::string& w) {
    for (auto& sp : body) {
      Stmt& x = *sp;
      for (EP* e : {&x.lhs, &x.rhs, &x.cond, &x.lo, &x.hi, &x.step, &x.ret}) rename_expr(*e, v, w);
      if (x.kind == Stmt::For && x.var == v) continue;   // an inner loop binds its own v
      rename_in(x.body, v, w);
      rename_in(x.els, v, w);
    }
  }

  // An array the sweep allocates itself at its top level (an HVP sweep's
  // tangent of a tape, `du_stack_d = Vector{Float64}(undef, length(du_stack))`)
  // becomes a trailing argument that the caller allocates: the library never
  // allocates. stade_<k>_locals gives the sizes.
  struct LocalArray {
    std::string name, type;
    EP size;
  };
  std::vector<LocalArray> locals_;
  void hoist_local_arrays() {
    std::vector<SP> kept;
    for (auto& sp : f_.body) {
      Stmt& s = *sp;
      if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Var && s.rhs->kind == Expr::Curly) {
        if (s.rhs->a.size() != 2) fail(s.line, "expected Vector{T}(undef, n)");
        locals_.push_back({s.lhs->s, s.rhs->s, s.rhs->a[1]});
        f_.params.push_back(s.lhs->s);
        arrays_.insert(s.lhs->s);
        if (s.rhs->s.find("Int") != std::string::npos) int_arrays_.insert(s.lhs->s);
        continue;
      }
      kept.push_back(sp);
    }
    if (locals_.empty()) return;
    f_.body = kept;
    link(f_.body, nullptr);
  }

  // stade_<k>_locals(<integer arguments>, <lengths of the arrays the sizes
  // read through length()>, sizes, dtypes): the sizes of the hoisted arrays
  std::string locals_src(std::string& mf) {
    if (locals_.empty()) {
      mf = "null";
      return "";
    }
    std::set<std::string> lens;
    for (auto& l : locals_)
      walk_expr(l.size, [&](const EP& x) {
        if (x->kind == Expr::Call && x->s == "length" && x->a.size() == 1 &&
            x->a[0]->kind == Expr::Var)
          lens.insert(x->a[0]->s);
      });
    std::ostringstream q;
    std::string ia, la;
    q << "extern \"C\" int64_t stade_" << f_.name << "_locals(";
    for (auto& p : f_.params)
      if (!arrays_.count(p) && ints_.count(p)) {
        q << "int64_t " << cname(p) << ", ";
        ia += std::string(ia.empty() ? "" : ", ") + jstr(p);
      }
    for (auto& p : f_.params)
      if (lens.count(p)) {
        q << "int64_t " << cname(p) << ", ";
        la += std::string(la.empty() ? "" : ", ") + jstr(p);
      }
    q << "int64_t* sizes, int* dtypes) {\n";
    std::set<std::string> loc(f_.params.begin(), f_.params.end());
    std::string ms;
    init_printing_ = true;
    for (size_t i = 0; i < locals_.size(); ++i) {
      const auto& l = locals_[i];
      const int code = l.type.find("Int") != std::string::npos ? 2 : (f32_ ? 1 : 0);
      q << "  if (sizes) sizes[" << i << "] = jl_imax((int64_t)0, (int64_t)("
        << cx(l.size, loc, 0) << "));\n";
      q << "  if (dtypes) dtypes[" << i << "] = " << code << ";\n";
      ms += std::string(ms.empty() ? "" : ", ") + "{\"name\": " + jstr(l.name) + ", \"dtype\": " +
            jstr(code == 2 ? "i64" : (code == 1 ? "f32" : "f64")) + "}";
    }
    init_printing_ = false;
    q << "  return " << locals_.size() << ";\n}\n";
    mf = "{\"symbol\": " + jstr("stade_" + f_.name + "_locals") + ", \"args\": [" + ia +
         "], \"length_args\": [" + la + "], \"arrays\": [" + ms + "]}";
    return q.str();
  }

  void run() {
    items_ = plan_body(f_.body);
    decide_storage();
    emit();
  }

 private:
  Func& f_;
  const Func* init_;
  bool f32_;
  // scatter -> gather rewrite of invertible accumulations (STADE_EMIT_GATHER=0: atomics)
  bool gather_ = !(std::getenv("STADE_EMIT_GATHER") && std::string(std::getenv("STADE_EMIT_GATHER")) == "0");
  std::string T_;
  std::set<std::string> params_, arrays_, ints_, int_arrays_, host_ints_, returned_;
  std::map<std::string, std::vector<EP>> dims_;
  std::vector<Unit> units_;
  std::vector<Item> items_;
  std::map<std::string, Storage> store_;
  std::map<std::string, int> fslot_, islot_;
  std::set<std::string> stacks_;
  std::set<std::string> tier_b_tables_;   // prefix_<stack>_<id> tables initstacks fills
  bool init_printing_ = false;          // printing initstacks: length(p) is the argument p
  std::string init_len_args_ = "[]";    // initstacks arguments passed as an array's length
  std::map<std::string, std::string> stack_type_;  // name -> "f" / "i"
  std::vector<std::string> decisions_;
  std::map<const Stmt*, std::string> red_sites_;   // accumulation -> block sum register
  std::set<int> blk_units_;                         // units whose kernel has block sums

  // ---- kinds: array / scalar, integer / float (the evidence shape_infer uses,
  // src/STADE.jl:936-958: loop variables, range bounds, div / mod arguments,
  // subscripts, comparisons against integer literals, then propagation)
  bool is_int_expr(const EP& e) const {
    switch (e->kind) {
      case Expr::Num:
        return e->int_lit;
      case Expr::Var:
        return ints_.count(e->s) > 0;
      case Expr::Ref:
        return int_arrays_.count(e->s) > 0;
      case Expr::Call: {
        const std::string& n = e->s;
        if (n == "div" || n == "mod" || n == "rem" || n == "Int" || n == "Int64" || n == "length" ||
            n == "mod1" || n == "fld" || n == "cld")
          return true;
        if (n == "max" || n == "min" || n == "abs" || n == "sign" || n == "ifelse") {
          for (size_t i = (n == "ifelse" ? 1 : 0); i < e->a.size(); ++i)
            if (!is_int_expr(e->a[i])) return false;
          return true;
        }
        return false;
      }
      case Expr::Bin:
        if (e->s == "/" ) return false;
        if (e->s == "==" || e->s == "!=" || e->s == "<" || e->s == ">" || e->s == "<=" ||
            e->s == ">=" || e->s == "&&" || e->s == "||")
          return true;
        return is_int_expr(e->a[0]) && is_int_expr(e->a[1]);
      case Expr::Un:
        return is_int_expr(e->a[0]);
      default:
        return false;
    }
  }

  void mark_int_leaves(const EP& e) {
    walk_expr(e, [&](const EP& x) {
      if (x->kind == Expr::Var) ints_.insert(x->s);
      if (x->kind == Expr::Call && (x->s == "div" || x->s == "mod" || x->s == "rem"))
        for (auto& c : x->a) mark_int_leaves(c);
    });
  }

  void infer_kinds() {
    walk_stmts(f_.body, [&](Stmt& s) {
      auto mark_arrays = [&](const EP& e) {
        walk_expr(e, [&](const EP& x) {
          if (x->kind == Expr::Ref) arrays_.insert(x->s);
        });
      };
      if (s.lhs) mark_arrays(s.lhs);
      if (s.rhs) mark_arrays(s.rhs);
      if (s.cond) mark_arrays(s.cond);
      if (s.ret) mark_arrays(s.ret);
      if (s.lo) mark_arrays(s.lo);
      if (s.hi) mark_arrays(s.hi);
      if (s.step) mark_arrays(s.step);
    });
    // direct evidence
    std::function<void(const EP&)> subscripts = [&](const EP& e) {
      walk_expr(e, [&](const EP& x) {
        if (x->kind == Expr::Ref)
          for (auto& i : x->a) {
            walk_expr(i, [&](const EP& y) {
              if (y->kind == Expr::Var && !arrays_.count(y->s)) ints_.insert(y->s);
              if (y->kind == Expr::Ref) int_arrays_.insert(y->s);   // an index table
            });
          }
        if (x->kind == Expr::Call && (x->s == "div" || x->s == "mod" || x->s == "rem"))
          for (auto& c : x->a) mark_int_leaves(c);
        if (x->kind == Expr::Bin && (x->s == "==" || x->s == "!=")) {
          const EP& l = x->a[0];
          const EP& r = x->a[1];
          if (r->kind == Expr::Num && r->int_lit && l->kind == Expr::Var) ints_.insert(l->s);
          if (l->kind == Expr::Num && l->int_lit && r->kind == Expr::Var) ints_.insert(r->s);
        }
      });
    };
    walk_stmts(f_.body, [&](Stmt& s) {
      if (s.kind == Stmt::For) {
        ints_.insert(s.var);
        mark_int_leaves(s.lo);
        mark_int_leaves(s.hi);
        if (s.step) mark_int_leaves(s.step);
      }
      for (const EP* e : {&s.lhs, &s.rhs, &s.cond, &s.lo, &s.hi, &s.step, &s.ret})
        if (*e) subscripts(*e);
    });
    // stacks declared Vector{Int64} by initstacks are integer arrays
    if (init_) {
      for (auto& s : init_->body)
        if (s->kind == Stmt::Assign && s->lhs->kind == Expr::Var && s->rhs->kind == Expr::Curly) {
          const std::string& ty = s->rhs->s;
          if (ty.find("Int") != std::string::npos) int_arrays_.insert(s->lhs->s);
        }
    }
    // propagation
    for (int it = 0; it < 16; ++it) {
      bool changed = false;
      walk_stmts(f_.body, [&](Stmt& s) {
        if (s.kind != Stmt::Assign) return;
        const std::string& name = s.lhs->s;
        bool lhs_int = s.lhs->kind == Expr::Var ? ints_.count(name) > 0 : int_arrays_.count(name) > 0;
        if (!lhs_int && is_int_expr(s.rhs)) {
          (s.lhs->kind == Expr::Var ? ints_ : int_arrays_).insert(name);
          changed = true;
        }
        if (lhs_int && s.rhs->kind == Expr::Var && !ints_.count(s.rhs->s)) {
          ints_.insert(s.rhs->s);
          changed = true;
        }
        // an integer assigned a sum / difference / product of variables and
        // integer literals (`w = m0 + i_x`): those variables are integers too
        if (lhs_int && s.rhs->kind == Expr::Bin) {
          bool arith = true;
          walk_expr(s.rhs, [&](const EP& x) {
            if (x->kind == Expr::Bin && x->s != "+" && x->s != "-" && x->s != "*") arith = false;
            if (x->kind == Expr::Num && !x->int_lit) arith = false;
            if (x->kind != Expr::Bin && x->kind != Expr::Num && x->kind != Expr::Var) arith = false;
          });
          if (arith)
            walk_expr(s.rhs, [&](const EP& x) {
              if (x->kind == Expr::Var && !arrays_.count(x->s) && !ints_.count(x->s)) {
                ints_.insert(x->s);
                changed = true;
              }
            });
        }
        if (lhs_int && s.rhs->kind == Expr::Ref && !int_arrays_.count(s.rhs->s)) {
          int_arrays_.insert(s.rhs->s);
          changed = true;
        }
      });
      if (!changed) break;
    }
    for (auto& a : arrays_) ints_.erase(a);
    // returned scalars
    walk_stmts(f_.body, [&](Stmt& s) {
      if (s.kind != Stmt::Return || !s.ret) return;
      std::vector<EP> items = s.ret->kind == Expr::Tuple ? s.ret->a : std::vector<EP>{s.ret};
      for (auto& e : items) {
        if (e->kind != Expr::Var || !params_.count(e->s) || arrays_.count(e->s) || ints_.count(e->s))
          fail(s.line, "a sweep may return only its float scalar arguments, found " + text(e));
        returned_.insert(e->s);
      }
    });
    // stacks: the trailing parameters initstacks returns, allocated there
    // (`Vector{T}(undef, n)`); a returned integer (`__len_m = length(m)`) is
    // an integer argument of the sweep
    if (init_) {
      std::set<std::string> allocated;
      for (auto& s : init_->body)
        if (s->kind == Stmt::Assign && s->lhs->kind == Expr::Var && s->rhs->kind == Expr::Curly)
          allocated.insert(s->lhs->s);
      // Tier-B prefix tables: filled by initstacks' sizing loop
      walk_stmts(init_->body, [&](Stmt& s) {
        if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Ref && s.lhs->s.rfind("prefix_", 0) == 0)
          tier_b_tables_.insert(s.lhs->s);
      });
      for (auto& s : init_->body)
        if (s->kind == Stmt::Return && s->ret) {
          std::vector<EP> items = s->ret->kind == Expr::Tuple ? s->ret->a : std::vector<EP>{s->ret};
          for (auto& e : items) {
            if (e->kind != Expr::Var) continue;
            if (allocated.count(e->s)) {
              stacks_.insert(e->s);
            } else if (params_.count(e->s)) {
              ints_.insert(e->s);
              arrays_.erase(e->s);
            }
          }
        }
    }
    for (auto& p : f_.params)
      if (!arrays_.count(p) && stacks_.count(p)) arrays_.insert(p);
  }

  void parse_dims(const std::string& spec) {
    size_t i = 0;
    while (i < spec.size()) {
      size_t j = spec.find(';', i);
      if (j == std::string::npos) j = spec.size();
      std::string item = spec.substr(i, j - i);
      i = j + 1;
      size_t eq = item.find('=');
      if (item.find_first_not_of(" \t") == std::string::npos) continue;
      if (eq == std::string::npos) fail(0, "dims entry '" + item + "' has no '='");
      std::string name = item.substr(0, eq);
      name.erase(std::remove_if(name.begin(), name.end(), ::isspace), name.end());
      // parse "d1, d2" through a one-line function wrapper
      Parser q(lex("function __d()\nreturn (" + item.substr(eq + 1) + ", 0)\nend\n"));
      auto funcs = q.file();
      EP tup = funcs[0].body[0]->ret;
      std::vector<EP> fs;
      for (size_t k = 0; k + 1 < tup->a.size(); ++k) fs.push_back(tup->a[k]);
      dims_[name] = fs;
    }
  }

  // leading dimensions of a multi-dimensional array: given, or the upper
  // bound of a `for v = 1:hi` whose variable is that subscript
  // The extent of a variable decoded from a flattened nest, the generators'
  // canonical form (`for idx = 1:A * n; i = div(idx - 1, n) + 1;
  // j = mod(idx - 1, n) + 1`): A for i, n for j. Null when v is not one.
  EP decoded_extent(const std::string& v) {
    std::map<std::string, std::vector<EP>> all;
    walk_stmts(f_.body, [&](Stmt& s) {
      if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Var) all[s.lhs->s].push_back(s.rhs);
    });
    auto one = [&](const std::string& name) -> EP {   // a temporary assigned one text
      auto f = all.find(name);
      if (f == all.end()) return nullptr;
      for (auto& e : f->second)
        if (text(e) != text(f->second[0])) return nullptr;
      return f->second[0];
    };
    // the top H of the range 1..H of loop variable idx (1:H or H:-1:1), one for all its loops
    auto top = [&](const std::string& idx) -> EP {
      EP h;
      bool ok = true;
      walk_stmts(f_.body, [&](Stmt& s) {
        if (s.kind != Stmt::For || s.var != idx) return;
        EP t;
        if (!s.step && s.lo->kind == Expr::Num && s.lo->s == "1") t = s.hi;
        else if (s.step && text(s.step) == "-1" && s.hi->kind == Expr::Num && s.hi->s == "1") t = s.lo;
        if (!t || (h && text(h) != text(t))) ok = false;
        if (t) h = t;
      });
      return ok ? h : nullptr;
    };
    auto extent = [&](const EP& r) -> EP {
      if (r->kind != Expr::Bin || r->s != "+" || r->a[1]->kind != Expr::Num || r->a[1]->s != "1")
        return nullptr;
      const EP& c = r->a[0];
      if (c->kind != Expr::Call || (c->s != "div" && c->s != "mod") || c->a.size() != 2)
        return nullptr;
      EP x = c->a[0];
      const EP& n = c->a[1];
      if (x->kind == Expr::Var) x = one(x->s);
      if (!x || x->kind != Expr::Bin || x->s != "-" || x->a[0]->kind != Expr::Var ||
          x->a[1]->kind != Expr::Num || x->a[1]->s != "1")
        return nullptr;
      EP h = top(x->a[0]->s);
      if (!h || h->kind != Expr::Bin || h->s != "*" || text(h->a[1]) != text(n)) return nullptr;
      return c->s == "div" ? h->a[0] : n;
    };
    auto it = all.find(v);
    if (it == all.end()) return nullptr;
    EP first;
    for (auto& r : it->second) {
      EP e = extent(r);
      if (!e || (first && text(first) != text(e))) return nullptr;
      first = e;
    }
    return first;
  }

  std::vector<EP> dims_of(const std::string& a, size_t rank, int line) {
    auto it = dims_.find(a);
    if (it != dims_.end()) {
      if (it->second.size() + 1 < rank) fail(line, "dims of " + a + " list too few extents");
      return it->second;
    }
    std::vector<EP> d(rank - 1);
    std::vector<std::set<std::string>> seen(rank - 1);
    walk_stmts(f_.body, [&](Stmt& s) {
      std::function<void(const EP&)> look = [&](const EP& e) {
        walk_expr(e, [&](const EP& x) {
          if (x->kind != Expr::Ref || x->s != a || x->a.size() != rank) return;
          for (size_t k = 0; k + 1 < rank; ++k) {
            if (x->a[k]->kind == Expr::Var) seen[k].insert(x->a[k]->s);
            if (d[k] || x->a[k]->kind != Expr::Var) continue;
            // find the enclosing loop of that variable
            for (Stmt* o = &s; o; o = o->owner)
              if (o->kind == Stmt::For && o->var == x->a[k]->s && !o->step &&
                  o->lo->kind == Expr::Num && o->lo->s == "1") {
                d[k] = o->hi;
                break;
              }
          }
        });
      };
      for (const EP* e : {&s.lhs, &s.rhs, &s.cond})
        if (*e) look(*e);
    });
    for (size_t k = 0; k + 1 < rank; ++k)
      for (auto& v : seen[k])
        if (!d[k]) d[k] = decoded_extent(v);
    for (size_t k = 0; k + 1 < rank; ++k)
      if (!d[k])
        fail(line, "cannot infer dimension " + std::to_string(k + 1) + " of " + a +
                       " (give it with dims, e.g. \"" + a + "=n_rows\")");
    dims_[a] = d;
    return d;
  }

  // ---- first reference of a scalar in a statement list -----------------------
  enum Ref3 { R_NONE, R_READ, R_WRITE };
  Ref3 first_ref(const std::vector<SP>& b, size_t from, size_t to, const std::string& v) {
    for (size_t i = from; i < to && i < b.size(); ++i) {
      Ref3 r = first_ref_stmt(*b[i], v);
      if (r != R_NONE) return r;
    }
    return R_NONE;
  }
  Ref3 first_ref_stmt(Stmt& s, const std::string& v) {
    switch (s.kind) {
      case Stmt::Assign:
        if (reads_scalar(s.rhs, v)) return R_READ;
        if (s.lhs->kind == Expr::Ref) {
          for (auto& i : s.lhs->a)
            if (reads_scalar(i, v)) return R_READ;
          return R_NONE;
        }
        return s.lhs->s == v ? R_WRITE : R_NONE;
      case Stmt::For: {
        if (reads_scalar(s.lo, v) || reads_scalar(s.hi, v) || (s.step && reads_scalar(s.step, v)))
          return R_READ;
        if (s.var == v) return R_WRITE;
        return first_ref(s.body, 0, s.body.size(), v) == R_READ ? R_READ : R_NONE;
      }
      case Stmt::While:
        if (reads_scalar(s.cond, v)) return R_READ;
        return first_ref(s.body, 0, s.body.size(), v) == R_READ ? R_READ : R_NONE;
      case Stmt::If: {
        if (reads_scalar(s.cond, v)) return R_READ;
        Ref3 a = first_ref(s.body, 0, s.body.size(), v);
        Ref3 b = first_ref(s.els, 0, s.els.size(), v);
        if (a == R_READ || b == R_READ) return R_READ;
        if (a == R_WRITE && b == R_WRITE) return R_WRITE;
        return R_NONE;
      }
      case Stmt::Return:
        return s.ret && reads_scalar(s.ret, v) ? R_READ : R_WRITE;  // nothing runs after
    }
    return R_NONE;
  }

  // Is v read after statement `st` before being rewritten?
  bool live_after(Stmt& st, const std::string& v) {
    Stmt* cur = &st;
    for (;;) {
      std::vector<SP>& b = *cur->in;
      Ref3 r = first_ref(b, cur->pos + 1, b.size(), v);
      if (r == R_READ) return true;
      if (r == R_WRITE) return false;
      Stmt* o = cur->owner;
      if (!o) return false;
      if (o->kind == Stmt::For || o->kind == Stmt::While) {
        if (first_ref(b, 0, cur->pos, v) == R_READ) return true;   // next iteration
        if (o->kind == Stmt::While && reads_scalar(o->cond, v)) return true;
      }
      cur = o;
    }
  }

  // The scalar always holds the literal c between iterations of every loop
  // that assigns it, and is set to c before anything reads it.
  bool convergent_constant(const std::string& v, std::string& c) {
    // first reference in the function: an unconditional top-level `v = literal`
    c.clear();
    for (auto& s : f_.body) {
      Ref3 r = first_ref_stmt(*s, v);
      if (r == R_READ) return false;
      if (r == R_WRITE) {
        if (s->kind != Stmt::Assign || s->rhs->kind != Expr::Num) return false;
        c = s->rhs->s;
        break;
      }
    }
    if (c.empty()) return false;
    bool ok = true;
    std::function<void(std::vector<SP>&, bool)> check = [&](std::vector<SP>& b, bool in_loop) {
      for (auto& s : b) {
        if (s->kind == Stmt::Assign && s->lhs->kind == Expr::Var && s->lhs->s == v && !in_loop &&
            !(s->rhs->kind == Expr::Num && s->rhs->s == c))
          ok = false;
        if (s->kind == Stmt::For || s->kind == Stmt::While) {
          bool assigns = false;
          walk_stmts(s->body, [&](Stmt& x) {
            if (x.kind == Stmt::Assign && x.lhs->kind == Expr::Var && x.lhs->s == v) assigns = true;
          });
          if (assigns) {
            // the last top-level statement referencing v must be `v = c`
            const Stmt* last = nullptr;
            for (auto& x : s->body)
              if (first_ref_stmt(*x, v) != R_NONE || mentions(*x, v)) last = x.get();
            if (!last || last->kind != Stmt::Assign || last->lhs->kind != Expr::Var ||
                last->lhs->s != v || last->rhs->kind != Expr::Num || last->rhs->s != c)
              ok = false;
          }
          check(s->body, true);
        } else if (s->kind == Stmt::If) {
          check(s->body, in_loop);
          check(s->els, in_loop);
        }
      }
    };
    check(f_.body, false);
    return ok;
  }

  bool mentions(Stmt& s, const std::string& v) {
    bool hit = false;
    std::vector<SP> one{std::shared_ptr<Stmt>(&s, [](Stmt*) {})};
    walk_stmts(one, [&](Stmt& x) {
      for (const EP* e : {&x.lhs, &x.rhs, &x.cond, &x.lo, &x.hi, &x.step, &x.ret})
        if (*e && reads_scalar(*e, v)) hit = true;
      if (x.kind == Stmt::For && x.var == v) hit = true;
    });
    return hit;
  }

  // ---- index classification --------------------------------------------------
  Cls classify(const EP& e, const std::string& v, const std::set<std::string>& varying,
               const std::set<std::string>& written, const std::map<std::string, EP>& defs,
               int depth) {
    Cls c;
    if (depth > 32) return c;
    switch (e->kind) {
      case Expr::Num:
        c.k = Cls::INV;
        return c;
      case Expr::Var: {
        if (e->s == v) {
          c.k = Cls::INJ;
          c.key = e->s;
          return c;
        }
        auto d = defs.find(e->s);
        if (d != defs.end()) return classify(d->second, v, varying, written, defs, depth + 1);
        c.k = varying.count(e->s) ? Cls::OTHER : Cls::INV;
        return c;
      }
      case Expr::Ref: {
        if (written.count(e->s)) return c;
        for (auto& i : e->a)
          if (classify(i, v, varying, written, defs, depth + 1).k != Cls::INV) return c;
        c.k = Cls::INV;
        return c;
      }
      case Expr::Call: {
        if ((e->s == "div" || e->s == "mod") && e->a.size() == 2) {
          Cls x = classify(e->a[0], v, varying, written, defs, depth + 1);
          Cls n = classify(e->a[1], v, varying, written, defs, depth + 1);
          if (x.k == Cls::INV && n.k == Cls::INV) {
            c.k = Cls::INV;
            return c;
          }
          if (x.k == Cls::INJ && n.k == Cls::INV) {
            c.k = e->s == "div" ? Cls::DIVP : Cls::MODP;
            c.key = canon(e->a[0], defs) + "|" + canon(e->a[1], defs);
            c.n = canon(e->a[1], defs);
          }
          return c;
        }
        for (auto& a : e->a)
          if (classify(a, v, varying, written, defs, depth + 1).k != Cls::INV) return c;
        c.k = Cls::INV;
        return c;
      }
      case Expr::Un: {
        Cls x = classify(e->a[0], v, varying, written, defs, depth + 1);
        if (e->s == "-" && (x.k == Cls::INV || x.k == Cls::INJ)) return x;
        return c;
      }
      case Expr::Bin: {
        Cls l = classify(e->a[0], v, varying, written, defs, depth + 1);
        Cls r = classify(e->a[1], v, varying, written, defs, depth + 1);
        if (e->s == "+" || e->s == "-") {
          if (l.k == Cls::INV && r.k == Cls::INV) return l;
          if (r.k == Cls::INV && l.k != Cls::OTHER) return l;
          if (l.k == Cls::INV && r.k != Cls::OTHER && e->s == "+") return r;
          if (l.k == Cls::INV && r.k == Cls::INJ) return r;
          if (e->s == "+" && ((l.k == Cls::MULDIV && r.k == Cls::MODP) ||
                              (l.k == Cls::MODP && r.k == Cls::MULDIV)) &&
              l.key == r.key) {
            c.k = Cls::INJ;
            c.key = l.key;
          }
          return c;
        }
        if (e->s == "*") {
          if (l.k == Cls::INV && r.k == Cls::INV) return l;
          if (l.k == Cls::INJ && r.k == Cls::INV) return l;
          if (l.k == Cls::INV && r.k == Cls::INJ) return r;
          if (l.k == Cls::DIVP && r.k == Cls::INV && canon(e->a[1], defs) == l.n) {
            c = l;
            c.k = Cls::MULDIV;
            return c;
          }
          if (r.k == Cls::DIVP && l.k == Cls::INV && canon(e->a[0], defs) == r.n) {
            c = r;
            c.k = Cls::MULDIV;
            return c;
          }
          return c;
        }
        if (l.k == Cls::INV && r.k == Cls::INV) return l;
        return c;
      }
      default:
        return c;
    }
  }

  std::string canon(const EP& e, const std::map<std::string, EP>& defs, int depth = 0) {
    if (depth > 32) return text(e);
    if (e->kind == Expr::Var) {
      auto d = defs.find(e->s);
      if (d != defs.end()) return canon(d->second, defs, depth + 1);
      return e->s;
    }
    if (e->kind == Expr::Num || e->kind == Expr::Curly) return e->s;
    std::string s = e->s + "(";
    for (auto& a : e->a) s += canon(a, defs, depth + 1) + ",";
    return s + ")";
  }

  bool injective(const std::vector<EP>& idx, const std::string& v,
                 const std::set<std::string>& varying, const std::set<std::string>& written,
                 const std::map<std::string, EP>& defs) {
    std::vector<Cls> cs;
    for (auto& i : idx) cs.push_back(classify(i, v, varying, written, defs, 0));
    for (auto& c : cs)
      if (c.k == Cls::INJ) return true;
    for (auto& a : cs)
      for (auto& b : cs)
        if (a.k == Cls::DIVP && b.k == Cls::MODP && a.key == b.key) return true;
    return false;
  }

  // A Tier-B tape slot (agen_tier_b_block_stmts, src/STADE.jl:5338-5380):
  // prefix_<stack>_<id>[f(v)] + g, the prefix table filled by initstacks and
  // indexed injectively by the thread variable, g varying only with loops
  // inside the iteration. The layout gives each iteration of the header loop
  // its own span of slots, so threads write disjoint slots.
  bool tier_b_slot(const std::vector<EP>& idx, const std::string& v,
                   const std::set<std::string>& varying, const std::set<std::string>& written,
                   const std::map<std::string, EP>& defs, const std::set<std::string>& inner) {
    if (idx.size() != 1) return false;
    std::vector<EP> terms;
    std::function<void(const EP&)> flat = [&](const EP& x) {
      if (x->kind == Expr::Bin && x->s == "+") {
        flat(x->a[0]);
        flat(x->a[1]);
      } else {
        terms.push_back(x);
      }
    };
    flat(subst(idx[0], defs));
    int n_prefix = 0;
    for (auto& t : terms) {
      if (t->kind == Expr::Ref && t->a.size() == 1 && tier_b_tables_.count(t->s) &&
          !written.count(t->s) && classify(t->a[0], v, varying, written, defs, 0).k == Cls::INJ) {
        ++n_prefix;
        continue;
      }
      bool ok = true;
      walk_expr(t, [&](const EP& y) {
        if (y->kind == Expr::Ref || (y->kind == Expr::Var && y->s == v) ||
            (y->kind == Expr::Var && varying.count(y->s) && !inner.count(y->s)))
          ok = false;
      });
      if (!ok) return false;
    }
    return n_prefix == 1;
  }

  // ---- loop plan ---------------------------------------------------------------
  struct Site {
    Stmt* st;
    bool write, accum;
    std::string idx;
    std::vector<EP> index;
  };

  // An accumulation `a[i] = a[i] + e`, `a[i] - e`, `e + a[i]`: the term (sign applied)
  static EP accum_term(const Stmt& s) {
    if (s.kind != Stmt::Assign || s.rhs->kind != Expr::Bin) return nullptr;
    const EP& l = s.rhs->a[0];
    const EP& r = s.rhs->a[1];
    auto same = [&](const EP& x) { return text(x) == text(s.lhs); };
    if ((s.rhs->s == "+" || s.rhs->s == "-") && same(l) && !reads_self(r, s.lhs)) {
      return s.rhs->s == "+" ? r : mk(Expr::Un, "-", {r});
    }
    if (s.rhs->s == "+" && same(r) && !reads_self(l, s.lhs)) return l;
    return nullptr;
  }
  static bool reads_self(const EP& e, const EP& lhs) {
    if (lhs->kind == Expr::Var) return reads_scalar(e, lhs->s);
    return reads_array(e, lhs->s);
  }

  // Private integer scalars of loop L assigned one expression (however often)
  // that does not read them: their definitions, to see through decoded indices.
  std::map<std::string, EP> int_defs(Stmt& L, const LoopPlan& p) {
    std::map<std::string, EP> defs;
    std::map<std::string, std::vector<EP>> rhs_of;
    walk_stmts(L.body, [&](Stmt& x) {
      if (x.kind == Stmt::Assign && x.lhs->kind == Expr::Var) rhs_of[x.lhs->s].push_back(x.rhs);
    });
    for (auto& [v, rs] : rhs_of) {
      auto pv = p.privates.find(v);
      if (pv == p.privates.end() || !pv->second.empty() || !ints_.count(v)) continue;
      bool same = true;
      for (auto& r : rs)
        if (text(r) != text(rs[0]) || reads_scalar(r, v)) same = false;
      if (same) defs[v] = rs[0];
    }
    return defs;
  }

  // ---- scatter -> gather ---------------------------------------------------------
  EP subst(const EP& e, const std::map<std::string, EP>& defs, int depth = 0) {
    if (!e) return e;
    if (e->kind == Expr::Var) {
      auto d = defs.find(e->s);
      if (d != defs.end() && depth < 32) return subst(d->second, defs, depth + 1);
      return e;
    }
    if (e->a.empty()) return e;
    auto c = std::make_shared<Expr>(*e);
    for (auto& x : c->a) x = subst(x, defs, depth + 1);
    return c;
  }
  static bool is_lit(const EP& e, long* v) {
    if (!e || e->kind != Expr::Num || !e->int_lit) return false;
    *v = std::stol(e->s);
    return true;
  }
  static bool is_var(const EP& e, const std::string& v) {
    return e->kind == Expr::Var && e->s == v;
  }
  static bool plus_one(const EP& e) {
    long one;
    return e->kind == Expr::Bin && e->s == "+" && is_lit(e->a[1], &one) && one == 1;
  }

  struct Coord {
    int axis;
    EP n;
    long shift;
  };
  // div(v - 1, n) + 1 (axis 0, the row) or mod(v - 1, n) + 1 (axis 1, the column)
  bool decode(const EP& e, const std::string& v, Coord& c) {
    if (!plus_one(e)) return false;
    const EP& f = e->a[0];
    if (f->kind != Expr::Call || (f->s != "div" && f->s != "mod") || f->a.size() != 2) return false;
    const EP& x = f->a[0];
    long k;
    if (!(x->kind == Expr::Bin && x->s == "-" && is_var(x->a[0], v) && is_lit(x->a[1], &k) &&
          k == 1))
      return false;
    c.axis = f->s == "div" ? 0 : 1;
    c.n = f->a[1];
    c.shift = 0;
    return true;
  }
  // a decoded coordinate, or its periodic shift mod(x + k, n) + 1 (by k + 1)
  bool coord(const EP& e, const std::string& v, Coord& c) {
    if (decode(e, v, c)) return true;
    if (!plus_one(e)) return false;
    const EP& f = e->a[0];
    if (f->kind != Expr::Call || f->s != "mod" || f->a.size() != 2) return false;
    EP base = f->a[0];
    long k = 0;
    Coord b;
    if (!decode(base, v, b)) {   // mod(x + k, n): strip the literal k
      if (!(base->kind == Expr::Bin && (base->s == "+" || base->s == "-") &&
            is_lit(base->a[1], &k)))
        return false;
      if (base->s == "-") k = -k;
      base = base->a[0];
      if (!decode(base, v, b)) return false;
    }
    if (text(b.n) != text(f->a[1])) return false;
    c = b;
    c.shift = k + 1;
    return true;
  }
  // the inverse of a target index: the identity, a constant offset, or a
  // periodic shift on the n x n grid that v = (i - 1) n + j flattens
  bool inverse_of(const EP& idx, const std::string& v, Inverse& inv) {
    long k;
    if (is_var(idx, v)) {
      inv.kind = Inverse::IDENT;
      return true;
    }
    if (idx->kind == Expr::Bin && (idx->s == "+" || idx->s == "-")) {
      if (is_var(idx->a[0], v) && is_lit(idx->a[1], &k)) {
        inv.kind = Inverse::OFFSET;
        inv.off = idx->s == "+" ? k : -k;
        return true;
      }
      if (idx->s == "+" && is_var(idx->a[1], v) && is_lit(idx->a[0], &k)) {
        inv.kind = Inverse::OFFSET;
        inv.off = k;
        return true;
      }
    }
    if (idx->kind == Expr::Bin && idx->s == "+") {
      for (int o = 0; o < 2; ++o) {
        const EP& prod = idx->a[o];
        const EP& cexp = idx->a[1 - o];
        if (prod->kind != Expr::Bin || prod->s != "*") continue;
        for (int q = 0; q < 2; ++q) {
          const EP& rm1 = prod->a[q];
          const EP& nn = prod->a[1 - q];
          long one;
          if (rm1->kind != Expr::Bin || rm1->s != "-" || !is_lit(rm1->a[1], &one) || one != 1)
            continue;
          Coord R, Cc;
          if (!coord(rm1->a[0], v, R) || !coord(cexp, v, Cc)) continue;
          if (R.axis != 0 || Cc.axis != 1 || text(R.n) != text(Cc.n) || text(R.n) != text(nn))
            continue;
          if (R.shift == 0 && Cc.shift == 0) {
            inv.kind = Inverse::IDENT;
            return true;
          }
          inv.kind = Inverse::PERIODIC2;
          inv.n = R.n;
          inv.sr = R.shift;
          inv.sc = Cc.shift;
          return true;
        }
      }
    }
    return false;
  }

  // Arrays that parallel loop L only accumulates into through invertible
  // indices: each becomes a gather (a thread per target element replays the
  // iterations that land on it, no atomics). The loop body must be
  // straight-line, and no array the loop writes may be read after its write,
  // so that a replay sees the values from before the loop.
  std::vector<Gather> plan_gather(Stmt& L, const LoopPlan& p) {
    std::vector<Gather> out;
    if (p.atomic_arrays.empty()) return out;
    for (auto& st : L.body)
      if (st->kind != Stmt::Assign) return out;
    long stepv = 1;
    if (L.step && !is_lit(L.step, &stepv)) return out;
    if (stepv != 1 && stepv != -1) return out;
    std::set<std::string> written;
    for (auto& st : L.body) {
      bool bad = false;
      auto chk = [&](const EP& e) {
        walk_expr(e, [&](const EP& y) {
          if (y->kind == Expr::Ref && written.count(y->s)) bad = true;
        });
      };
      chk(st->rhs);
      if (st->lhs->kind == Expr::Ref)
        for (auto& i : st->lhs->a) chk(i);
      if (bad) return out;
      if (st->lhs->kind == Expr::Ref && !accum_term(*st)) written.insert(st->lhs->s);
    }
    const std::map<std::string, EP> defs = int_defs(L, p);
    for (auto& a : p.atomic_arrays) {
      if (int_arrays_.count(a)) continue;
      Gather g;
      g.array = a;
      bool ok = true;
      for (auto& st : L.body) {
        if (st->lhs->kind != Expr::Ref || st->lhs->s != a) continue;
        EP term = accum_term(*st);
        Inverse inv;
        if (!term || st->lhs->a.size() != 1 ||
            !inverse_of(subst(st->lhs->a[0], defs), L.var, inv)) {
          ok = false;
          break;
        }
        if (inv.kind == Inverse::PERIODIC2) {   // the loop covers the whole grid
          const EP& lo = stepv == 1 ? L.lo : L.hi;
          const EP& hi = stepv == 1 ? L.hi : L.lo;
          long one;
          const std::string cn = canon(inv.n, {});
          if (!is_lit(lo, &one) || one != 1 || canon(hi, {}) != "*(" + cn + "," + cn + ",)") {
            ok = false;
            break;
          }
        }
        g.parts.push_back({st.get(), term, inv});
      }
      if (ok && !g.parts.empty()) out.push_back(g);
    }
    return out;
  }

  LoopPlan plan_loop(Stmt& L) {
    LoopPlan p;
    std::set<std::string> assigned, inner_vars{L.var}, written;
    bool has_while = false, has_return = false;
    walk_stmts(L.body, [&](Stmt& s) {
      if (s.kind == Stmt::Assign) {
        if (s.lhs->kind == Expr::Var) assigned.insert(s.lhs->s);
        else written.insert(s.lhs->s);
      }
      if (s.kind == Stmt::For) inner_vars.insert(s.var);
      if (s.kind == Stmt::While) has_while = true;
      if (s.kind == Stmt::Return) has_return = true;
    });
    if (has_while) {
      p.why = "holds a while loop";
      return p;
    }
    if (has_return) {
      p.why = "holds a return";
      return p;
    }
    if (!host_int_expr(L.lo) || !host_int_expr(L.hi) || (L.step && !host_int_expr(L.step))) {
      p.why = "bounds are not integer arguments";
      return p;
    }
    std::set<std::string> varying = assigned;
    varying.insert(inner_vars.begin(), inner_vars.end());
    // scalars
    for (const auto& s : assigned) {
      if (inner_vars.count(s)) continue;
      bool is_param = params_.count(s) > 0;
      // private: no path through an iteration reads it before writing it
      if (!is_param && first_ref(L.body, 0, L.body.size(), s) != R_READ && !live_after(L, s)) {
        p.privates[s] = "";
        continue;
      }
      std::string c;
      if (!is_param && convergent_constant(s, c)) {
        p.privates[s] = c;
        continue;
      }
      // reduction: only `s = s +- e`, never read otherwise
      int n_acc = 0, n_reads = 0;
      bool only_acc = true;
      walk_stmts(L.body, [&](Stmt& x) {
        if (x.kind == Stmt::Assign && x.lhs->kind == Expr::Var && x.lhs->s == s) {
          if (accum_term(x)) ++n_acc;
          else only_acc = false;
        }
        for (const EP* e : {&x.rhs, &x.cond, &x.lo, &x.hi, &x.step})
          if (*e) walk_expr(*e, [&](const EP& y) {
              if (y->kind == Expr::Var && y->s == s) ++n_reads;
            });
        if (x.lhs && x.lhs->kind == Expr::Ref)
          for (auto& i : x.lhs->a)
            walk_expr(i, [&](const EP& y) {
              if (y->kind == Expr::Var && y->s == s) ++n_reads;
            });
      });
      if (only_acc && n_acc > 0 && n_reads == n_acc && !ints_.count(s)) {
        p.reductions.insert(s);
        continue;
      }
      p.why = "scalar " + s + " carries a value from one iteration to the next";
      return p;
    }
    // private integer definitions used to see through decoded indices
    std::map<std::string, EP> defs = int_defs(L, p);
    // arrays
    std::map<std::string, std::vector<Site>> sites;
    walk_stmts(L.body, [&](Stmt& s) {
      auto reads = [&](const EP& e, const EP& skip) {
        walk_expr(e, [&](const EP& x) {
          if (x->kind == Expr::Ref && x.get() != skip.get())
            sites[x->s].push_back({&s, false, false, idx_text(x), x->a});
        });
      };
      if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Ref) {
        EP term = accum_term(s);
        EP self;
        if (term) self = (text(s.rhs->a[0]) == text(s.lhs)) ? s.rhs->a[0] : s.rhs->a[1];
        sites[s.lhs->s].push_back({&s, true, term != nullptr, idx_text(s.lhs), s.lhs->a});
        for (auto& i : s.lhs->a) reads(i, nullptr);
        reads(s.rhs, self);
      } else {
        for (const EP* e : {&s.rhs, &s.cond, &s.lo, &s.hi, &s.step})
          if (*e) reads(*e, nullptr);
      }
    });
    for (auto& [a, ss] : sites) {
      bool any_write = false, all_acc = true, same = true, any_read = false;
      for (auto& x : ss) {
        if (x.write) {
          any_write = true;
          if (!x.accum) all_acc = false;
        } else {
          any_read = true;
        }
        if (x.idx != ss[0].idx) same = false;
      }
      if (!any_write) continue;
      if (same && injective(ss[0].index, L.var, varying, written, defs)) continue;
      if (same && tier_b_slot(ss[0].index, L.var, varying, written, defs, inner_vars)) continue;
      if (all_acc && !any_read) {
        p.atomic_arrays.insert(a);
        continue;
      }
      p.why = "array " + a + " is written and read at elements other threads may touch";
      return p;
    }
    p.parallel = true;
    return p;
  }

  std::string idx_text(const EP& r) {
    std::string s;
    for (auto& i : r->a) s += text(i) + ";";
    return s;
  }

  // ---- host integers -----------------------------------------------------------
  bool host_int_expr(const EP& e) {
    bool ok = true;
    walk_expr(e, [&](const EP& x) {
      if (x->kind == Expr::Ref) ok = false;
      if (x->kind == Expr::Var && !host_ints_.count(x->s) &&
          !(params_.count(x->s) && ints_.count(x->s)))
        ok = false;
      if (x->kind == Expr::Num && !x->int_lit) ok = false;
      if (x->kind == Expr::Call && !(x->s == "div" || x->s == "mod" || x->s == "max" ||
                                     x->s == "min" || x->s == "rem" || x->s == "abs"))
        ok = false;
      if (x->kind == Expr::Bin && x->s == "/") ok = false;
    });
    return ok;
  }

  bool assigned_only_at_top(const std::string& v) {
    bool ok = true;
    walk_stmts(f_.body, [&](Stmt& s) {
      if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Var && s.lhs->s == v && s.owner) ok = false;
      if (s.kind == Stmt::For && s.var == v) ok = false;
    });
    return ok;
  }

  bool has_parallel_loop(std::vector<SP>& b) {
    for (auto& s : b) {
      if (s->kind == Stmt::For) {
        bool added = host_ints_.insert(s->var).second;
        bool par = plan_loop(*s).parallel;
        bool inner = !par && host_int_expr(s->lo) && host_int_expr(s->hi) &&
                     (!s->step || host_int_expr(s->step)) && has_parallel_loop(s->body);
        if (added) host_ints_.erase(s->var);
        if (par || inner) return true;
      }
      if (s->kind == Stmt::If && host_int_expr(s->cond) &&
          (has_parallel_loop(s->body) || has_parallel_loop(s->els)))
        return true;
    }
    return false;
  }

  std::vector<Item> plan_body(std::vector<SP>& b) {
    std::vector<Item> items;
    std::vector<SP> seq;
    auto flush = [&]() {
      if (seq.empty()) return;
      Unit u;
      u.par = false;
      u.stmts = seq;
      u.id = (int)units_.size();
      units_.push_back(u);
      Item it;
      it.kind = Item::Kernel;
      it.unit = u.id;
      items.push_back(it);
      for (auto& s : seq) record_seq(*s, "in a one-thread kernel with its neighbours");
      seq.clear();
    };
    for (auto& s : b) {
      switch (s->kind) {
        case Stmt::Assign:
          if (s->lhs->kind == Expr::Var && ints_.count(s->lhs->s) && !s->owner &&
              assigned_only_at_top(s->lhs->s) && host_int_expr(s->rhs)) {
            flush();
            host_ints_.insert(s->lhs->s);
            Item it;
            it.kind = Item::HostAssign;
            it.st = s;
            items.push_back(it);
          } else {
            seq.push_back(s);
          }
          break;
        case Stmt::For: {
          LoopPlan p = plan_loop(*s);
          if (p.parallel) {
            flush();
            std::vector<Gather> gs = gather_ ? plan_gather(*s, p) : std::vector<Gather>{};
            SP rest;
            LoopPlan prest;
            if (!gs.empty()) {
              // the loop without the gathered accumulations
              rest = std::make_shared<Stmt>(*s);
              rest->body.clear();
              for (auto& st : s->body) {
                bool part = false;
                for (auto& g : gs)
                  for (auto& q : g.parts) part = part || q.st == st.get();
                if (!part) rest->body.push_back(st);
              }
              prest = plan_loop(*rest);
              if (!prest.parallel) gs.clear();
            }
            if (!gs.empty()) {
              Unit ug;
              ug.par = ug.gather = true;
              ug.gathers = gs;
              ug.stmts = {s};
              ug.plan = p;
              ug.id = (int)units_.size();
              units_.push_back(ug);
              Item ig;
              ig.kind = Item::Kernel;
              ig.unit = ug.id;
              items.push_back(ig);
              std::vector<std::string> names;
              for (auto& g : gs) names.push_back(g.array);
              decisions_.push_back(json_decision(*s, "gather", "", {}, {}, {}, names));
              if (!rest->body.empty()) {
                Unit u;
                u.par = true;
                u.stmts = {rest};
                u.plan = prest;
                u.id = (int)units_.size();
                units_.push_back(u);
                Item it;
                it.kind = Item::Kernel;
                it.unit = u.id;
                items.push_back(it);
                record_par(*rest, prest);
              }
              break;
            }
            Unit u;
            u.par = true;
            u.stmts = {s};
            u.plan = p;
            u.id = (int)units_.size();
            units_.push_back(u);
            Item it;
            it.kind = Item::Kernel;
            it.unit = u.id;
            items.push_back(it);
            record_par(*s, p);
            break;
          }
          bool host_loop = false;
          if (host_int_expr(s->lo) && host_int_expr(s->hi) && (!s->step || host_int_expr(s->step))) {
            host_ints_.insert(s->var);
            host_loop = has_parallel_loop(s->body);
            if (!host_loop) host_ints_.erase(s->var);
          }
          if (host_loop) {
            flush();
            decisions_.push_back(json_decision(*s, "host", p.why, {}, {}, {}));
            Item it;
            it.kind = Item::HostFor;
            it.st = s;
            it.a = plan_body(s->body);
            items.push_back(it);
          } else {
            decisions_.push_back(json_decision(*s, "sequential", p.why, {}, {}, {}));
            mark_inner_sequential(s->body);
            seq.push_back(s);
          }
          break;
        }
        case Stmt::If:
          if (host_int_expr(s->cond) && (has_parallel_loop(s->body) || has_parallel_loop(s->els))) {
            flush();
            Item it;
            it.kind = Item::HostIf;
            it.st = s;
            it.a = plan_body(s->body);
            it.b = plan_body(s->els);
            items.push_back(it);
          } else {
            mark_inner_sequential(s->body);
            mark_inner_sequential(s->els);
            seq.push_back(s);
          }
          break;
        case Stmt::While:
          mark_inner_sequential(s->body);
          seq.push_back(s);
          break;
        case Stmt::Return: {
          flush();
          if (s->owner || s->pos + 1 != s->in->size())
            fail(s->line, "only a final top-level return is supported");
          Item it;
          it.kind = Item::Return;
          it.st = s;
          items.push_back(it);
          break;
        }
      }
    }
    flush();
    return items;
  }

  void mark_inner_sequential(std::vector<SP>& b) {
    for (auto& s : b)
      if (s->kind == Stmt::For)
        decisions_.push_back(json_decision(*s, "sequential", "inside a sequential region", {}, {}, {}));
  }
  void record_seq(Stmt&, const char*) {}
  void record_par(Stmt& s, const LoopPlan& p) {
    std::vector<std::string> priv, red, atom;
    for (auto& [k, v] : p.privates) priv.push_back(v.empty() ? k : k + "=" + v);
    red.assign(p.reductions.begin(), p.reductions.end());
    atom.assign(p.atomic_arrays.begin(), p.atomic_arrays.end());
    decisions_.push_back(json_decision(s, "parallel", "", priv, red, atom));
  }

  static std::string jstr(const std::string& s) {
    std::string o = "\"";
    for (char c : s) {
      if (c == '"' || c == '\\') o += '\\';
      if (c == '\n') {
        o += "\\n";
        continue;
      }
      o += c;
    }
    return o + "\"";
  }
  static std::string jlist(const std::vector<std::string>& v) {
    std::string o = "[";
    for (size_t i = 0; i < v.size(); ++i) o += (i ? ", " : "") + jstr(v[i]);
    return o + "]";
  }
  std::string json_decision(Stmt& s, const std::string& mode, const std::string& why,
                            const std::vector<std::string>& priv,
                            const std::vector<std::string>& red,
                            const std::vector<std::string>& atom,
                            const std::vector<std::string>& gathered = {}) {
    std::string loop = "for " + s.var + " = " + text(s.lo) + ":" +
                       (s.step ? text(s.step) + ":" : "") + text(s.hi);
    return "{\"line\": " + std::to_string(s.line) + ", \"loop\": " + jstr(loop) +
           ", \"mode\": " + jstr(mode) + ", \"why\": " + jstr(why) +
           ", \"private\": " + jlist(priv) + ", \"reductions\": " + jlist(red) +
           ", \"atomics\": " + jlist(atom) + ", \"gathered\": " + jlist(gathered) + "}";
  }

  // ---- storage -----------------------------------------------------------------
  void unit_refs(Unit& u) {
    auto visit_expr = [&](const EP& e) {
      walk_expr(e, [&](const EP& x) {
        if (x->kind == Expr::Var && !arrays_.count(x->s)) u.scalars.insert(x->s);
        if (x->kind == Expr::Ref) u.arrays.insert(x->s);
      });
    };
    walk_stmts(u.stmts, [&](Stmt& s) {
      for (const EP* e : {&s.lhs, &s.rhs, &s.cond, &s.lo, &s.hi, &s.step, &s.ret})
        if (*e) visit_expr(*e);
      if (s.kind == Stmt::For) u.inner_vars.insert(s.var);
    });
    // dims of multi-dimensional arrays are read too
    for (auto& a : std::set<std::string>(u.arrays)) {
      auto it = dims_.find(a);
      if (it != dims_.end())
        for (auto& d : it->second) visit_expr(d);
    }
    for (auto& v : u.inner_vars) u.scalars.erase(v);
  }

  void decide_storage() {
    // make sure dims of every multi-dimensional array are known first
    walk_stmts(f_.body, [&](Stmt& s) {
      for (const EP* e : {&s.lhs, &s.rhs, &s.cond})
        if (*e)
          walk_expr(*e, [&](const EP& x) {
            if (x->kind == Expr::Ref && x->a.size() > 1) dims_of(x->s, x->a.size(), s.line);
          });
    });
    std::map<std::string, int> n_units;
    for (auto& u : units_) {
      unit_refs(u);
      for (auto& s : u.scalars) ++n_units[s];
    }
    // float arguments the sweep never assigns (alpha) go to the kernels by value
    std::set<std::string> assigned;
    walk_stmts(f_.body, [&](Stmt& s) {
      if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Var) assigned.insert(s.lhs->s);
      if (s.kind == Stmt::For) assigned.insert(s.var);
    });
    for (auto& p : f_.params) {
      if (arrays_.count(p)) continue;
      if (ints_.count(p)) store_[p] = S_HOSTINT;
      else if (!assigned.count(p) && !returned_.count(p)) store_[p] = S_FPARAM;
      else store_[p] = S_FBOX;
    }
    for (auto& h : host_ints_) store_[h] = S_HOSTINT;
    for (auto& u : units_) {
      for (auto& s : u.scalars) {
        if (store_.count(s)) continue;
        if (u.par && (u.plan.privates.count(s))) continue;   // private: a register
        if (n_units[s] == 1 && !(u.par && u.plan.reductions.count(s))) {
          continue;   // local to its one unit
        }
        store_[s] = ints_.count(s) ? S_IBOX : S_FBOX;
      }
    }
    for (auto& [s, st] : store_) {
      if (st == S_FBOX) fslot_[s] = (int)fslot_.size();
      if (st == S_IBOX) islot_[s] = (int)islot_.size();
    }
  }

  // ---- C++ expression printing -------------------------------------------------
  std::string cname(const std::string& v) { return "j_" + v; }
  std::set<std::string> fd_avail_;   // divisors with a jl_fd argument in the kernel being printed
  std::string fast_divisor(const EP& d, const std::set<std::string>& locals) {
    if (!d || d->kind != Expr::Var || locals.count(d->s) || !fd_avail_.count(d->s)) return "";
    return "fd_" + d->s;
  }
  size_t fstride() const { return f32_ ? 32 : 16; }   // elements per 128-byte line

  std::string scalar_ref(const std::string& v, const std::set<std::string>& locals) {
    if (locals.count(v)) return cname(v);
    auto it = store_.find(v);
    if (it == store_.end()) return cname(v);
    switch (it->second) {
      case S_HOSTINT:
      case S_LOCAL:
      case S_FPARAM:
        return cname(v);
      case S_FBOX:
        return "g_fbox[" + std::to_string(fslot_.at(v) * fstride()) + "]";
      case S_IBOX:
        return "g_ibox[" + std::to_string(islot_.at(v) * 16) + "]";
    }
    return cname(v);
  }

  std::string flit(const std::string& s) {
    std::string t = s;
    if (t.find_first_of(".eE") == std::string::npos) t += ".0";
    if (t.back() == '.') t += "0";
    return f32_ ? "(" + t + "f)" : "(" + t + ")";
  }

  std::string offset(const EP& r, const std::set<std::string>& locals, int line) {
    if (r->a.size() == 1) return "(" + cx(r->a[0], locals, line) + " - 1)";
    std::vector<EP> d = dims_of(r->s, r->a.size(), line);
    std::string o = "(" + cx(r->a[0], locals, line) + " - 1)";
    std::string stride;
    for (size_t k = 1; k < r->a.size(); ++k) {
      std::string dk = "(int64_t)(" + cx(d[k - 1], locals, line) + ")";
      stride = stride.empty() ? dk : stride + " * " + dk;
      o += " + (" + cx(r->a[k], locals, line) + " - 1) * " + stride;
    }
    return "(" + o + ")";
  }

  std::string cx(const EP& e, const std::set<std::string>& locals, int line) {
    switch (e->kind) {
      case Expr::Num:
        return e->int_lit ? "((int64_t)" + e->s + ")" : flit(e->s);
      case Expr::Var:
        if (arrays_.count(e->s)) fail(line, "array " + e->s + " used as a scalar");
        return scalar_ref(e->s, locals);
      case Expr::Ref:
        if (!arrays_.count(e->s)) fail(line, e->s + " is indexed but not an array argument");
        return "p_" + e->s + "[" + offset(e, locals, line) + "]";
      case Expr::Un:
        return "(" + e->s + cx(e->a[0], locals, line) + ")";
      case Expr::Tuple:
      case Expr::Curly:
        fail(line, "unexpected " + text(e));
      case Expr::Bin: {
        const std::string& op = e->s;
        std::string l = cx(e->a[0], locals, line), r = cx(e->a[1], locals, line);
        if (op == "/") return "((" + T_ + ")" + l + " / (" + T_ + ")" + r + ")";
        const std::string fd = fast_divisor(e->a[1], locals);
        if (op == "÷") return fd.empty() ? "jl_div(" + l + ", " + r + ")" : "jl_divf(" + l + ", " + r + ", " + fd + ")";
        if (op == "%" && is_int_expr(e))
          return fd.empty() ? "jl_rem(" + l + ", " + r + ")" : "jl_remf(" + l + ", " + r + ", " + fd + ")";
        if (op == "%") return "fmod(" + l + ", " + r + ")";
        if (op == "^") {
          const EP& x = e->a[1];
          bool ib = is_int_expr(e->a[0]);
          if (x->kind == Expr::Num && x->int_lit) {
            long k = std::stol(x->s);
            if (k == 2) return "jl_sq(" + l + ")";
            if (k == 3) return "jl_cube(" + l + ")";
            if (k == 1) return "(" + l + ")";
            if (k == 0) return ib ? "((int64_t)1)" : "((" + T_ + ")1)";
            if (k == -1 && !ib) return "((" + T_ + ")1 / (" + T_ + ")" + l + ")";
            if (ib && k > 0) return "jl_ipow(" + l + ", " + x->s + ")";
          }
          return "jl_pow((" + T_ + ")" + l + ", (" + T_ + ")" + r + ")";
        }
        return "(" + l + " " + op + " " + r + ")";
      }
      case Expr::Call: {
        const std::string& n = e->s;
        if (n == "length" && init_printing_ && e->a.size() == 1 && e->a[0]->kind == Expr::Var)
          return cname(e->a[0]->s);   // the caller passes the array's length
        std::vector<std::string> a;
        for (auto& x : e->a) a.push_back(cx(x, locals, line));
        auto need = [&](size_t k) {
          if (a.size() != k) fail(line, n + " takes " + std::to_string(k) + " arguments");
        };
        bool all_int = is_int_expr(e);
        if (n == "div" || n == "mod" || n == "rem" || n == "fld" || n == "cld" || n == "mod1") {
          need(2);
          if (!is_int_expr(e->a[0]) || !is_int_expr(e->a[1]))
            fail(line, n + " of a float is not supported");
          const std::string fd = fast_divisor(e->a[1], locals);
          if (!fd.empty() && (n == "div" || n == "mod" || n == "rem"))
            return "jl_" + n + "f(" + a[0] + ", " + a[1] + ", " + fd + ")";
          return "jl_" + n + "(" + a[0] + ", " + a[1] + ")";
        }
        if (n == "max" || n == "min") {
          if (a.size() < 2) fail(line, n + " takes at least 2 arguments");
          std::string acc = a[0];
          for (size_t k = 1; k < a.size(); ++k)
            acc = (all_int ? "jl_i" + n : "jl_" + n) + "(" +
                  (all_int ? acc : "(" + T_ + ")" + acc) + ", " +
                  (all_int ? a[k] : "(" + T_ + ")" + a[k]) + ")";
          return acc;
        }
        if (n == "abs" || n == "sign") {
          need(1);
          return all_int ? "jl_i" + n + "(" + a[0] + ")" : "jl_" + n + "((" + T_ + ")" + a[0] + ")";
        }
        static const std::set<std::string> fns = {"sqrt", "exp", "log", "tanh", "sin", "cos", "tan",
                                                  "sinh", "cosh", "asin", "acos", "atan", "log2",
                                                  "log10", "exp2", "expm1", "log1p", "cbrt"};
        if (fns.count(n)) {
          need(1);
          return "jl_" + n + "((" + T_ + ")" + a[0] + ")";
        }
        if (n == "Float64" || n == "Float32" || n == "float") {
          need(1);
          return "((" + T_ + ")" + a[0] + ")";
        }
        if (n == "Int" || n == "Int64") {
          need(1);
          return "((int64_t)" + a[0] + ")";
        }
        if (n == "ifelse") {
          need(3);
          return "((" + a[0] + ") ? (" + a[1] + ") : (" + a[2] + "))";
        }
        if (n == "zero" || n == "one") {
          need(1);
          std::string v = n == "zero" ? "0" : "1";
          return is_int_expr(e->a[0]) ? "((int64_t)" + v + ")" : "((" + T_ + ")" + v + ")";
        }
        fail(line, "function " + n + " is not supported");
      }
    }
    fail(line, "unsupported expression");
  }

  std::string ctype(const std::string& v) { return ints_.count(v) ? "int64_t" : T_; }

  // ---- statement printing (device code) ---------------------------------------
  void stmts(std::ostringstream& o, const std::vector<SP>& b, const std::set<std::string>& locals,
             const Unit& u, int ind) {
    for (auto& s : b) stmt(o, *s, locals, u, ind);
  }

  // Deferred array stores of a straight-line parallel body: a store waits in
  // registers until a later statement reads (or atomically updates) the same
  // array, or the body ends, so the loads of an iteration issue before its
  // stores (the arrays are distinct __restrict__ arguments). Measured on a
  // tape-restore loop (u = tape; ub read then zeroed; unb += ...): 745 us in
  // statement order, 120 us with the stores deferred.
  // A store whose value does not come from the load of the same address
  // (the generated `__oldb = xb[i]; xb[i] = 0.0`) still issues at once and,
  // with that load in flight, held a stencil adjoint loop at 2980 us instead
  // of 650 us: its value is given a dependence on the loaded register
  // (jl_after with the kernel argument z_, which is 0), so it issues after the
  // load returns and stores the same bits.
  struct Pending {
    std::string array, off, val;
  };
  std::vector<Pending>* pending_ = nullptr;
  int pending_n_ = 0;
  std::map<std::string, std::string> loaded_;   // "A[offset]" -> register loaded from it

  void flush_pending(std::ostringstream& o, const std::string& pad, const std::set<std::string>& arrays,
                     bool all) {
    if (!pending_) return;
    std::vector<Pending> keep;
    for (auto& p : *pending_) {
      if (all || arrays.count(p.array))
        o << pad << "p_" << p.array << "[" << p.off << "] = " << p.val << ";\n";
      else
        keep.push_back(p);
    }
    *pending_ = keep;
  }

  void stmt(std::ostringstream& o, Stmt& s, const std::set<std::string>& locals, const Unit& u,
            int ind) {
    std::string pad(ind, ' ');
    if (pending_ && s.kind == Stmt::Assign) {
      std::set<std::string> reads;
      walk_expr(s.rhs, [&](const EP& y) {
        if (y->kind == Expr::Ref) reads.insert(y->s);
      });
      if (s.lhs->kind == Expr::Ref) {
        for (auto& i : s.lhs->a)
          walk_expr(i, [&](const EP& y) {
            if (y->kind == Expr::Ref) reads.insert(y->s);
          });
        const bool plain = !red_sites_.count(&s) && !(u.par && u.plan.atomic_arrays.count(s.lhs->s));
        if (!plain) reads.insert(s.lhs->s);
      }
      flush_pending(o, pad, reads, false);
      if (s.lhs->kind == Expr::Ref && !red_sites_.count(&s) &&
          !(u.par && u.plan.atomic_arrays.count(s.lhs->s))) {
        const std::string& a = s.lhs->s;
        const std::string n = std::to_string(pending_n_++);
        const std::string ty = int_arrays_.count(a) ? "int64_t" : T_;
        const std::string off = offset(s.lhs, locals, s.line);
        std::string val = "(" + ty + ")" + cx(s.rhs, locals, s.line);
        auto ld = loaded_.find(a + "[" + off + "]");
        if (ld != loaded_.end() && reads.empty()) {
          bool uses = false;
          walk_expr(s.rhs, [&](const EP& y) {
            if (y->kind == Expr::Var && cname(y->s) == ld->second) uses = true;
          });
          if (!uses) val = "jl_after(" + val + ", jl_bits(" + ld->second + ") & z_)";
        }
        o << pad << "const int64_t so" << n << "_ = " << off << ";\n";
        o << pad << "const " << ty << " sv" << n << "_ = " << val << ";\n";
        pending_->push_back({a, "so" + n + "_", "sv" + n + "_"});
        return;
      }
      if (s.lhs->kind == Expr::Var && s.rhs->kind == Expr::Ref && locals.count(s.lhs->s) &&
          arrays_.count(s.rhs->s))
        loaded_[s.rhs->s + "[" + offset(s.rhs, locals, s.line) + "]"] = cname(s.lhs->s);
    }
    switch (s.kind) {
      case Stmt::Assign: {
        if (s.lhs->kind == Expr::Var) {
          const std::string& v = s.lhs->s;
          if (red_sites_.count(&s)) {
            o << pad << red_sites_[&s] << " += (" << T_ << ")" << cx(accum_term(s), locals, s.line)
              << ";\n";
            return;
          }
          if (u.par && u.plan.reductions.count(v)) {
            EP term = accum_term(s);
            o << pad << "jl_atomic_add(&" << scalar_ref(v, {}) << ", (" << T_ << ")"
              << cx(term, locals, s.line) << ");\n";
            return;
          }
          if (!locals.count(v) && store_.count(v) && store_[v] == S_HOSTINT)
            fail(s.line, "integer " + v + " is assigned on the device and on the host");
          o << pad << scalar_ref(v, locals) << " = " << cast_to(v, cx(s.rhs, locals, s.line))
            << ";\n";
          return;
        }
        const std::string& a = s.lhs->s;
        if (red_sites_.count(&s)) {
          o << pad << red_sites_[&s] << " += (" << T_ << ")" << cx(accum_term(s), locals, s.line)
            << ";\n";
          return;
        }
        if (u.par && u.plan.atomic_arrays.count(a)) {
          EP term = accum_term(s);
          std::string ty = int_arrays_.count(a) ? "unsigned long long" : T_;
          if (int_arrays_.count(a))
            o << pad << "atomicAdd((unsigned long long*)&p_" << a << "[" << offset(s.lhs, locals, s.line)
              << "], (unsigned long long)(" << cx(term, locals, s.line) << "));\n";
          else
            o << pad << "jl_atomic_add(&p_" << a << "[" << offset(s.lhs, locals, s.line) << "], ("
              << T_ << ")" << cx(term, locals, s.line) << ");\n";
          (void)ty;
          return;
        }
        o << pad << "p_" << a << "[" << offset(s.lhs, locals, s.line) << "] = "
          << (int_arrays_.count(a) ? "(int64_t)" : "(" + T_ + ")") << cx(s.rhs, locals, s.line)
          << ";\n";
        return;
      }
      case Stmt::For: {
        std::string v = cname(s.var);
        std::string st = s.step ? cx(s.step, locals, s.line) : "((int64_t)1)";
        bool lit = !s.step || (s.step->kind == Expr::Num && s.step->int_lit);
        bool neg = s.step && lit && s.step->s[0] == '-';
        o << pad << "{\n";
        o << pad << "  const int64_t lo_ = " << cx(s.lo, locals, s.line) << ", hi_ = "
          << cx(s.hi, locals, s.line) << ", st_ = " << st << ";\n";
        std::string cond = lit ? (neg ? v + " >= hi_" : v + " <= hi_")
                               : "(st_ > 0 ? " + v + " <= hi_ : " + v + " >= hi_)";
        o << pad << "  for (int64_t " << v << " = lo_; " << cond << "; " << v << " += st_) {\n";
        std::set<std::string> inner = locals;
        inner.insert(s.var);
        stmts(o, s.body, inner, u, ind + 4);
        o << pad << "  }\n" << pad << "}\n";
        return;
      }
      case Stmt::While:
        o << pad << "while (" << cx(s.cond, locals, s.line) << ") {\n";
        stmts(o, s.body, locals, u, ind + 2);
        o << pad << "}\n";
        return;
      case Stmt::If:
        o << pad << "if (" << cx(s.cond, locals, s.line) << ") {\n";
        stmts(o, s.body, locals, u, ind + 2);
        o << pad << "}";
        if (!s.els.empty()) {
          o << " else {\n";
          stmts(o, s.els, locals, u, ind + 2);
          o << pad << "}";
        }
        o << "\n";
        return;
      case Stmt::Return:
        fail(s.line, "return inside a loop or branch is not supported");
    }
  }

  std::string cast_to(const std::string& v, const std::string& e) {
    return "(" + ctype(v) + ")" + e;
  }

  // ---- kernels -----------------------------------------------------------------
  struct KArgs {
    std::vector<std::string> decl, pass;
  };

  KArgs kernel_args(const Unit& u) {
    KArgs k;
    for (auto& p : f_.params) {
      if (arrays_.count(p) && u.arrays.count(p)) {
        std::string ty = int_arrays_.count(p) ? "int64_t" : T_;
        k.decl.push_back(ty + "* __restrict__ p_" + p);
        k.pass.push_back("p_" + p);
      }
    }
    for (auto& s : u.scalars) {
      auto it = store_.find(s);
      if (it != store_.end() && it->second == S_HOSTINT) {
        k.decl.push_back("int64_t " + cname(s));
        k.pass.push_back(cname(s));
      }
      if (it != store_.end() && it->second == S_FPARAM) {
        k.decl.push_back(T_ + " " + cname(s));
        k.pass.push_back(cname(s));
      }
    }
    for (auto& d : divisors(u)) {
      k.decl.push_back("jl_fd fd_" + d);
      k.pass.push_back("jl_fd_make(" + cname(d) + ")");
    }
    return k;
  }

  // host-integer scalars a unit divides by (div / mod / rem, ÷, %, and the
  // periodic inverses of its gathers)
  std::set<std::string> divisors(const Unit& u) {
    std::set<std::string> d;
    auto host_int = [&](const EP& e) {
      if (!e || e->kind != Expr::Var) return;
      auto it = store_.find(e->s);
      if (it != store_.end() && it->second == S_HOSTINT && u.scalars.count(e->s)) d.insert(e->s);
    };
    auto visit = [&](const EP& e) {
      walk_expr(e, [&](const EP& x) {
        if (x->kind == Expr::Call && (x->s == "div" || x->s == "mod" || x->s == "rem") &&
            x->a.size() == 2)
          host_int(x->a[1]);
        if (x->kind == Expr::Bin && (x->s == "÷" || x->s == "%") && is_int_expr(x)) host_int(x->a[1]);
      });
    };
    walk_stmts(u.stmts, [&](Stmt& s) {
      for (const EP* e : {&s.lhs, &s.rhs, &s.cond, &s.lo, &s.hi, &s.step, &s.ret})
        if (*e) visit(*e);
    });
    for (auto& g : u.gathers)
      for (auto& q : g.parts)
        if (q.inv.kind == Inverse::PERIODIC2) host_int(q.inv.n);
    return d;
  }

  // v_ = the iteration whose accumulation lands on jt_
  std::string inverse_src(const Inverse& inv, const std::set<std::string>& locals, int line) {
    switch (inv.kind) {
      case Inverse::IDENT:
        return "v_ = jt_;";
      case Inverse::OFFSET:
        return "v_ = jt_ - (" + std::to_string(inv.off) + ");";
      case Inverse::PERIODIC2: {
        const std::string n = "(int64_t)(" + cx(inv.n, locals, line) + ")";
        const std::string fd = fast_divisor(inv.n, locals);
        const std::string dv = fd.empty() ? "jl_div(jt_ - 1, nn_)" : "jl_divf(jt_ - 1, nn_, " + fd + ")";
        const std::string md = fd.empty() ? "jl_mod" : "jl_modf";
        const std::string fa = fd.empty() ? "" : ", " + fd;
        return "{ const int64_t nn_ = " + n + "; const int64_t q_ = " + dv +
               "; const int64_t r_ = " + md + "(q_ - (" + std::to_string(inv.sr) + "), nn_" + fa +
               "), c_ = " + md + "((jt_ - 1 - q_ * nn_) - (" + std::to_string(inv.sc) + "), nn_" + fa +
               "); v_ = r_ * nn_ + c_ + 1; }";
      }
    }
    return "v_ = jt_;";
  }
  static std::string inv_key(const Inverse& v) {
    return std::to_string((int)v.kind) + ":" + std::to_string(v.off) + ":" +
           std::to_string(v.sr) + ":" + std::to_string(v.sc);
  }

  std::string gather_src(const Unit& u) {
    std::ostringstream o;
    KArgs k = kernel_args(u);
    Stmt& L = *u.stmts[0];
    o << "// " << text_loop(L) << "  (line " << L.line
      << "): gather, a thread per target element replays the iterations that land on it\n";
    o << "__global__ void stade_k" << u.id << "(int64_t jlo_, int64_t n_, int64_t vlo_, int64_t vhi_";
    for (auto& d : k.decl) o << ", " << d;
    o << ") {\n";
    o << "  const int64_t tid_ = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;\n";
    o << "  if (tid_ >= n_) return;\n";
    o << "  const int64_t jt_ = jlo_ + tid_;\n";
    std::set<std::string> base;
    for (auto& sc : u.scalars) {
      if (u.plan.privates.count(sc) || u.plan.reductions.count(sc) || sc == L.var) continue;
      auto it = store_.find(sc);
      if (it == store_.end()) fail(L.line, "scalar " + sc + " is read but never set");
      if (it->second == S_FBOX || it->second == S_IBOX) {
        o << "  const " << ctype(sc) << " " << cname(sc) << " = " << scalar_ref(sc, {}) << ";\n";
        base.insert(sc);
      }
    }
    for (auto& g : u.gathers) {
      o << "  {\n    " << T_ << " acc_ = p_" << g.array << "[jt_ - 1];\n    bool any_ = false;\n";
      // parts grouped by inverse, each group one replay of the body up to its last part
      std::vector<std::string> keys;
      for (auto& q : g.parts)
        if (std::find(keys.begin(), keys.end(), inv_key(q.inv)) == keys.end())
          keys.push_back(inv_key(q.inv));
      for (auto& key : keys) {
        const GatherPart* first = nullptr;
        std::set<const Stmt*> mine;
        for (auto& q : g.parts)
          if (inv_key(q.inv) == key) {
            if (!first) first = &q;
            mine.insert(q.st);
          }
        std::set<std::string> locals = base;
        locals.insert(L.var);
        o << "    {\n      int64_t v_;\n      " << inverse_src(first->inv, locals, L.line) << "\n";
        o << "      if (v_ >= vlo_ && v_ <= vhi_) {\n        any_ = true;\n";
        o << "        const int64_t " << cname(L.var) << " = v_;\n";
        for (auto& [v, init] : u.plan.privates) {
          const std::string iv = init.empty() ? "0" : (ints_.count(v) ? init : flit(init));
          o << "        " << ctype(v) << " " << cname(v) << " = " << cast_to(v, iv) << ";\n";
          locals.insert(v);
        }
        size_t left = mine.size();
        for (auto& st : L.body) {
          if (!left) break;
          if (mine.count(st.get())) {
            const GatherPart* q = nullptr;
            for (auto& x : g.parts)
              if (x.st == st.get()) q = &x;
            o << "        acc_ += (" << T_ << ")" << cx(q->term, locals, st->line) << ";\n";
            --left;
          } else if (st->lhs->kind == Expr::Var && u.plan.privates.count(st->lhs->s)) {
            o << "        " << cname(st->lhs->s) << " = "
              << cast_to(st->lhs->s, cx(st->rhs, locals, st->line)) << ";\n";
          }
        }
        o << "      }\n    }\n";
      }
      o << "    if (any_) p_" << g.array << "[jt_ - 1] = acc_;\n  }\n";
    }
    o << "}\n";
    return o.str();
  }

  std::string kernel_src(const Unit& u) {
    fd_avail_ = divisors(u);
    std::string r = u.gather ? gather_src(u) : kernel_body_src(u);
    fd_avail_.clear();
    return r;
  }

  std::string kernel_body_src(const Unit& u) {
    std::ostringstream o, decl;   // decl: device arrays the kernel needs, before it
    KArgs k = kernel_args(u);
    std::string name = "stade_k" + std::to_string(u.id);
    if (u.par) {
      Stmt& L = *u.stmts[0];
      o << "// " << text_loop(L) << "  (line " << L.line << "): thread per iteration\n";
      o << "__global__ void " << name << "(int64_t lo_, int64_t st_, int64_t n_, int64_t z_";
      for (auto& d : k.decl) o << ", " << d;
      o << ") {\n";
      // accumulations into one loop-invariant target from one site: a block
      // sum per block, the blocks' sums added in block order by the last block
      // (the generated loss and scalar-adjoint sums)
      std::vector<std::pair<std::string, std::string>> blk;   // register, target
      red_sites_.clear();
      {
        std::set<std::string> varying{L.var}, written;
        walk_stmts(L.body, [&](Stmt& x) {
          if (x.kind == Stmt::Assign && x.lhs->kind == Expr::Var) varying.insert(x.lhs->s);
          if (x.kind == Stmt::Assign && x.lhs->kind == Expr::Ref) written.insert(x.lhs->s);
          if (x.kind == Stmt::For) varying.insert(x.var);
        });
        std::map<std::string, std::vector<Stmt*>> sites;
        walk_stmts(L.body, [&](Stmt& x) {
          if (x.kind != Stmt::Assign || !accum_term(x)) return;
          const std::string& nm = x.lhs->s;
          if (x.lhs->kind == Expr::Var ? u.plan.reductions.count(nm) > 0
                                       : u.plan.atomic_arrays.count(nm) > 0)
            sites[nm].push_back(&x);
          else if (x.lhs->kind == Expr::Ref && u.plan.atomic_arrays.count(nm))
            sites[nm].push_back(&x);
        });
        for (auto& [nm, ss] : sites) {
          if (ss.size() != 1) continue;
          Stmt* x = ss[0];
          if (x->lhs->kind == Expr::Ref) {
            if (int_arrays_.count(nm)) continue;
            bool inv = true;
            for (auto& i : x->lhs->a)
              if (classify(i, L.var, varying, written, {}, 0).k != Cls::INV) inv = false;
            if (!inv) continue;
          }
          const std::string reg = "red" + std::to_string(blk.size()) + "_";
          red_sites_[x] = reg;
          blk.push_back({reg, x->lhs->kind == Expr::Var
                                  ? "&" + scalar_ref(nm, {})
                                  : "&p_" + nm + "[" + offset(x->lhs, {}, x->line) + "]"});
        }
      }
      // a kernel with block sums strides over the iterations with a grid the
      // SMs hold at once, so that one slot per resident block remains
      const std::string ind = blk.empty() ? "  " : "    ";
      std::ostringstream pv, rd;
      std::set<std::string> locals{L.var};
      for (auto& [v, init] : u.plan.privates) {
        std::string iv = init.empty() ? "0" : (ints_.count(v) ? init : flit(init));
        pv << ind << ctype(v) << " " << cname(v) << " = " << cast_to(v, iv) << ";\n";
        locals.insert(v);
      }
      // scalars only read: from their box (or by value), once
      for (auto& s : u.scalars) {
        if (locals.count(s) || u.plan.reductions.count(s)) continue;
        auto it = store_.find(s);
        if (it == store_.end()) fail(L.line, "scalar " + s + " is read but never set");
        if (it->second == S_FBOX || it->second == S_IBOX) {
          rd << "  const " << ctype(s) << " " << cname(s) << " = " << scalar_ref(s, {}) << ";\n";
          locals.insert(s);
        }
      }
      if (blk.empty()) {
        o << "  const int64_t tid_ = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;\n";
        o << "  if (tid_ >= n_) return;\n";
        o << "  const int64_t " << cname(L.var)
          << " = lo_ + (STADE_ASC && st_ < 0 ? n_ - 1 - tid_ : tid_) * st_;\n";
        o << pv.str() << rd.str();
      } else {
        blk_units_.insert(u.id);
        for (auto& [reg, tgt] : blk) o << "  " << T_ << " " << reg << " = 0;\n";
        o << rd.str();
        o << "  for (int64_t tid_ = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; tid_ < n_;\n"
          << "       tid_ += (int64_t)gridDim.x * blockDim.x) {\n";
        o << "    const int64_t " << cname(L.var)
          << " = lo_ + (STADE_ASC && st_ < 0 ? n_ - 1 - tid_ : tid_) * st_;\n";
        o << pv.str();
      }
      for (auto& v : u.inner_vars) locals.insert(v);
      locals.erase(L.var);
      locals.insert(L.var);
      std::set<std::string> body_locals = locals;
      bool straight = true;
      for (auto& st : L.body)
        if (st->kind != Stmt::Assign) straight = false;
      std::vector<Pending> pend;
      if (straight) pending_ = &pend;
      loaded_.clear();
      if (blk.empty()) {
        stmts(o, L.body, body_locals, u, 2);
        flush_pending(o, "  ", {}, true);
      } else {
        stmts(o, L.body, body_locals, u, 4);
        flush_pending(o, "    ", {}, true);
        o << "  }\n";
        // each block's sums go to a slot of their own; the last block to
        // finish adds the slots to the targets in block order (no float
        // atomics: the same sums in the same order on every call)
        const std::string parts = "stade_bpart" + std::to_string(u.id) + "_";
        const std::string ticket = "stade_bticket" + std::to_string(u.id) + "_";
        decl << "__device__ " << T_ << " " << parts << "[" << blk.size() << " * STADE_MAX_RES_BLOCKS];\n"
             << "__device__ unsigned " << ticket << " = 0;\n";
        o << "#ifdef STADE_EMIT_HOST\n";
        for (auto& [reg, tgt] : blk) o << "  jl_block_add(" << tgt << ", " << reg << ");\n";
        o << "#else\n";
        for (size_t j = 0; j < blk.size(); ++j)
          o << "  jl_block_part(" << parts << " + " << j << " * STADE_MAX_RES_BLOCKS, "
            << blk[j].first << ");\n";
        o << "  if (jl_block_last(&" << ticket << ")) {\n";
        for (size_t j = 0; j < blk.size(); ++j)
          o << "    jl_block_finish(" << blk[j].second << ", " << parts << " + " << j
            << " * STADE_MAX_RES_BLOCKS);\n";
        o << "    if (threadIdx.x == 0) " << ticket << " = 0;\n  }\n";
        o << "#endif\n";
      }
      pending_ = nullptr;
      red_sites_.clear();
      o << "}\n";
    } else {
      o << "// statements at line " << u.stmts[0]->line << ": one thread, in order\n";
      o << "__global__ void " << name << "(";
      for (size_t i = 0; i < k.decl.size(); ++i) o << (i ? ", " : "") << k.decl[i];
      o << ") {\n";
      o << "  if (blockIdx.x != 0 || threadIdx.x != 0) return;\n";
      std::set<std::string> locals;
      for (auto& s : u.scalars) {
        if (store_.count(s)) continue;
        o << "  " << ctype(s) << " " << cname(s) << " = 0;\n";
        locals.insert(s);
      }
      stmts(o, u.stmts, locals, u, 2);
      o << "}\n";
    }
    return decl.str() + o.str();
  }

  std::string text_loop(Stmt& s) {
    return "for " + s.var + " = " + text(s.lo) + ":" + (s.step ? text(s.step) + ":" : "") +
           text(s.hi);
  }

  void host_items(std::ostringstream& o, const std::vector<Item>& items, int ind) {
    std::string pad(ind, ' ');
    for (auto& it : items) {
      switch (it.kind) {
        case Item::HostAssign:
          o << pad << cname(it.st->lhs->s) << " = " << cx(it.st->rhs, {}, it.st->line) << ";\n";
          break;
        case Item::HostFor: {
          Stmt& s = *it.st;
          std::string v = cname(s.var);
          o << pad << "{\n" << pad << "  const int64_t lo_ = " << cx(s.lo, {}, s.line)
            << ", hi_ = " << cx(s.hi, {}, s.line)
            << ", st_ = " << (s.step ? cx(s.step, {}, s.line) : "((int64_t)1)") << ";\n";
          o << pad << "  for (int64_t " << v << " = lo_; st_ > 0 ? " << v << " <= hi_ : " << v
            << " >= hi_; " << v << " += st_) {\n";
          host_items(o, it.a, ind + 4);
          o << pad << "  }\n" << pad << "}\n";
          break;
        }
        case Item::HostIf:
          o << pad << "if (" << cx(it.st->cond, {}, it.st->line) << ") {\n";
          host_items(o, it.a, ind + 2);
          o << pad << "} else {\n";
          host_items(o, it.b, ind + 2);
          o << pad << "}\n";
          break;
        case Item::Kernel: {
          const Unit& u = units_[it.unit];
          KArgs k = kernel_args(u);
          std::string name = "stade_k" + std::to_string(u.id);
          if (u.gather) {
            Stmt& L = *u.stmts[0];
            long lo_off = 0, hi_off = 0;
            for (auto& g : u.gathers)
              for (auto& q : g.parts)
                if (q.inv.kind == Inverse::OFFSET) {
                  lo_off = std::min(lo_off, q.inv.off);
                  hi_off = std::max(hi_off, q.inv.off);
                }
            o << pad << "{\n" << pad << "  const int64_t a_ = " << cx(L.lo, {}, L.line)
              << ", b_ = " << cx(L.hi, {}, L.line) << ";\n";
            o << pad << "  const int64_t vlo_ = a_ < b_ ? a_ : b_, vhi_ = a_ < b_ ? b_ : a_;\n";
            o << pad << "  const int64_t jlo_ = vlo_ + (" << lo_off << "), jhi_ = vhi_ + (" << hi_off
              << ");\n";
            o << pad << "  if (jhi_ >= jlo_ && jl_trip(a_, " << (L.step ? cx(L.step, {}, L.line) : "((int64_t)1)")
              << ", b_) > 0) {\n";
            o << pad << "    const int64_t n_ = jhi_ - jlo_ + 1;\n";
            o << pad << "    STADE_LAUNCH(" << name
              << ", (unsigned)((n_ + 255) / 256), 256, s_, jlo_, n_, vlo_, vhi_";
            for (auto& p : k.pass) o << ", " << p;
            o << ");\n" << pad << "    STADE_GEN_CHECK();\n" << pad << "  }\n" << pad << "}\n";
            break;
          }
          if (u.par) {
            Stmt& L = *u.stmts[0];
            o << pad << "{\n" << pad << "  const int64_t lo_ = " << cx(L.lo, {}, L.line)
              << ", hi_ = " << cx(L.hi, {}, L.line)
              << ", st_ = " << (L.step ? cx(L.step, {}, L.line) : "((int64_t)1)") << ";\n";
            o << pad << "  const int64_t n_ = jl_trip(lo_, st_, hi_);\n";
            o << pad << "  if (n_ > 0) {\n";
            std::string grid = "(unsigned)((n_ + 255) / 256)";
            if (blk_units_.count(u.id)) {
              o << pad << "    static int cap_ = 0;\n" << pad
                << "    if (cap_ == 0) cap_ = stade_resident_blocks((const void*)" << name << ");\n";
              grid = "(unsigned)((n_ + 255) / 256 < cap_ ? (n_ + 255) / 256 : cap_)";
              o << pad << "    if (cap_ > STADE_MAX_RES_BLOCKS) cap_ = STADE_MAX_RES_BLOCKS;\n";
            }
            o << pad << "    STADE_LAUNCH(" << name << ", " << grid << ", 256, s_, lo_, st_, n_, (int64_t)0";
            for (auto& p : k.pass) o << ", " << p;
            o << ");\n" << pad << "    STADE_GEN_CHECK();\n" << pad << "  }\n" << pad << "}\n";
          } else {
            o << pad << "STADE_LAUNCH(" << name << ", 1, 1, s_";
            for (auto& p : k.pass) o << ", " << p;
            o << ");\n" << pad << "STADE_GEN_CHECK();\n";
          }
          break;
        }
        case Item::Return:
          break;
      }
    }
  }

  // ---- whole file --------------------------------------------------------------
  void emit() {
    std::ostringstream o;
    o << "// Generated by stade_emit from " << f_.name << " (STADE.jl generated sweep).\n"
      << "// Loop decisions are listed in the manifest.\n";
    o << prelude();
    o << "namespace {\n";
    // one 128-byte line per boxed scalar: a scalar every thread reads (alpha)
    // must not share a line with one the blocks add into (alphab)
    o << "__device__ " << T_ << " g_fbox[" << std::max<size_t>(1, fslot_.size()) * fstride()
      << "];\n";
    o << "__device__ int64_t g_ibox[" << std::max<size_t>(1, islot_.size()) * 16 << "];\n";
    // box initialisation kernel: the float scalar arguments
    std::vector<std::string> fparams;
    for (auto& p : f_.params)
      if (!arrays_.count(p) && store_.at(p) == S_FBOX) fparams.push_back(p);
    o << "__global__ void stade_k_init(";
    for (size_t i = 0; i < fparams.size(); ++i) o << (i ? ", " : "") << T_ << " v" << i;
    if (fparams.empty()) o << "int unused_";
    o << ") {\n";
    for (size_t i = 0; i < fparams.size(); ++i)
      o << "  g_fbox[" << fslot_.at(fparams[i]) * fstride() << "] = v" << i << ";\n";
    if (fparams.empty()) o << "  (void)unused_;\n";
    o << "}\n";
    for (auto& u : units_) o << kernel_src(u);
    o << "}  // namespace\n\n";
    // host function
    o << "extern \"C\" int stade_" << f_.name << "(";
    std::vector<std::string> decl;
    std::string mf_args;
    for (auto& p : f_.params) {
      std::string kind;
      if (arrays_.count(p)) {
        bool ia = int_arrays_.count(p) > 0;
        decl.push_back((ia ? "int64_t* p_" : T_ + "* p_") + p);
        kind = ia ? "array_int" : "array_float";
      } else if (ints_.count(p)) {
        decl.push_back("int64_t " + cname(p));
        kind = "scalar_int";
      } else if (returned_.count(p)) {
        decl.push_back(T_ + "* h_" + p);
        kind = "scalar_float_inout";
      } else {
        decl.push_back(T_ + " " + cname(p));
        kind = "scalar_float";
      }
      bool local = false;
      for (auto& l : locals_) local = local || l.name == p;
      mf_args += std::string(mf_args.empty() ? "" : ", ") + "{\"name\": " + jstr(p) +
                 ", \"kind\": " + jstr(kind) + ", \"stack\": " +
                 (stacks_.count(p) ? "true" : "false") + ", \"local\": " +
                 (local ? "true" : "false") + "}";
    }
    for (size_t i = 0; i < decl.size(); ++i) o << decl[i] << ", ";
    o << "void* stream) {\n";
    o << "  cudaStream_t s_ = (cudaStream_t)stream;\n  (void)s_;\n";
    o << "  STADE_CLEAR_ERROR();   // a failure before this call is not this call's\n";
    for (auto& h : host_ints_)
      if (!params_.count(h)) o << "  int64_t " << cname(h) << " = 0;\n";
    o << "  STADE_LAUNCH(stade_k_init, 1, 1, s_";
    for (auto& p : fparams) o << ", " << (returned_.count(p) ? "*h_" + p : cname(p));
    if (fparams.empty()) o << ", 0";
    o << ");\n  STADE_GEN_CHECK();\n";
    host_items(o, items_, 2);
    if (!returned_.empty()) {
      o << "  " << T_ << " box_[" << fslot_.size() * fstride() << "];\n";
      o << "  if (stade_box_read(box_, g_fbox, sizeof(box_), s_) != 0) return 3;\n";
      for (auto& r : returned_)
        o << "  *h_" << r << " = box_[" << fslot_.at(r) * fstride() << "];\n";
    }
    o << "  return 0;\n}\n\n";
    o << "extern \"C\" int64_t stade_" << f_.name << "_launches(void) { return stade_launches_; }\n\n";
    std::string mf_locals;
    o << locals_src(mf_locals);
    // initstacks
    std::string mf_stacks = "[]", init_sym = "null", init_args = "[]";
    if (init_) {
      o << initstacks_src(mf_stacks, init_args);
      init_sym = jstr("stade_" + init_->name);
    }
    cu = o.str();
    std::string ret;
    for (auto& r : returned_) ret += std::string(ret.empty() ? "" : ", ") + jstr(r);
    // order returned scalars as the return statement lists them
    std::vector<std::string> ret_order;
    walk_stmts(f_.body, [&](Stmt& s) {
      if (s.kind == Stmt::Return && s.ret) {
        std::vector<EP> items = s.ret->kind == Expr::Tuple ? s.ret->a : std::vector<EP>{s.ret};
        for (auto& e : items) ret_order.push_back(e->s);
      }
    });
    std::string dec;
    for (auto& d : decisions_) dec += std::string(dec.empty() ? "" : ",\n  ") + d;
    manifest = "{\"function\": " + jstr(f_.name) + ", \"symbol\": " + jstr("stade_" + f_.name) +
               ", \"precision\": " + jstr(f32_ ? "f32" : "f64") + ", \"args\": [" + mf_args +
               "], \"returns\": " + jlist(ret_order) + ", \"initstacks\": {\"symbol\": " + init_sym +
               ", \"args\": " + init_args + ", \"length_args\": " + init_len_args_ +
               ", \"stacks\": " + mf_stacks + "}, \"locals\": " + mf_locals + ", \"kernels\": " +
               std::to_string(units_.size()) + ", \"loops\": [\n  " + dec + "]}\n";
  }

  // initstacks_<k> as a host function whose statements run in order: the
  // closed-form stack sizes of agen_indexed_layout (src/STADE.jl:4917), or
  // the Tier-B sizing loop of agen_tier_b_block_stmts (src/STADE.jl:5338-5380)
  // with its prefix / value tables and running totals. Per returned item:
  //   a stack it allocates and does not fill: its size, dtype 0 / 1 (float,
  //   the sweep's precision) or 2 (Int64), zero-filled by the caller;
  //   a table it fills: its size, dtype 4 (Int64) or 5 (float), and its
  //   contents copied into fill[i] when the caller passes a buffer there;
  //   an integer (a total, __len_m): its value in sizes[i], dtype 3.
  std::string initstacks_src(std::string& mf_stacks, std::string& init_args) {
    const Func& F = *init_;
    std::map<std::string, std::string> alloc_ty;   // allocated array -> Vector{T}
    std::set<std::string> written, scalars, loop_vars;
    walk_stmts(F.body, [&](Stmt& s) {
      if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Var) {
        if (s.rhs->kind == Expr::Curly) {
          if (s.rhs->a.size() != 2) fail(s.line, "expected Vector{T}(undef, n)");
          alloc_ty[s.lhs->s] = s.rhs->s;
        } else {
          scalars.insert(s.lhs->s);
        }
      } else if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Ref) {
        written.insert(s.lhs->s);
      } else if (s.kind == Stmt::For) {
        loop_vars.insert(s.var);
      } else if (s.kind != Stmt::If && s.kind != Stmt::While && s.kind != Stmt::Return) {
        fail(s.line, "unsupported statement in " + F.name);
      }
    });
    for (auto& w : written)
      if (!alloc_ty.count(w)) fail(F.line, F.name + " writes " + w + ", which it does not allocate");
    // arrays of the initstacks body, as cx prints them (p_<name>)
    for (auto& [a, ty] : alloc_ty) {
      arrays_.insert(a);
      if (ty.find("Int") != std::string::npos) int_arrays_.insert(a);
      else int_arrays_.erase(a);
    }
    // scalar types: integer unless some assignment gives a float
    for (auto& p : F.params) ints_.insert(p);
    for (auto& v : loop_vars) ints_.insert(v);
    for (auto& v : scalars) ints_.insert(v);
    std::set<std::string> floats;
    for (bool changed = true; changed;) {
      changed = false;
      walk_stmts(F.body, [&](Stmt& s) {
        if (s.kind == Stmt::Assign && s.lhs->kind == Expr::Var && s.rhs->kind != Expr::Curly &&
            !floats.count(s.lhs->s) && !is_int_expr(s.rhs)) {
          floats.insert(s.lhs->s);
          ints_.erase(s.lhs->s);
          changed = true;
        }
      });
    }
    std::set<std::string> locals(F.params.begin(), F.params.end());
    locals.insert(scalars.begin(), scalars.end());
    locals.insert(loop_vars.begin(), loop_vars.end());

    std::ostringstream q;
    q << "extern \"C\" int64_t stade_" << F.name << "(";
    std::string ia, la;
    std::set<std::string> len_params;
    walk_stmts(F.body, [&](Stmt& s) {
      for (const EP* e : {&s.lhs, &s.rhs, &s.cond, &s.lo, &s.hi, &s.step})
        if (*e)
          walk_expr(*e, [&](const EP& x) {
            if (x->kind == Expr::Call && x->s == "length" && x->a.size() == 1 &&
                x->a[0]->kind == Expr::Var)
              len_params.insert(x->a[0]->s);
          });
    });
    for (auto& p : F.params) {
      q << "int64_t " << cname(p) << ", ";
      ia += std::string(ia.empty() ? "" : ", ") + jstr(p);
      if (len_params.count(p)) la += std::string(la.empty() ? "" : ", ") + jstr(p);
    }
    init_len_args_ = "[" + la + "]";
    init_args = "[" + ia + "]";
    q << "int64_t* sizes, int* dtypes, void* const* fill) {\n";
    q << "  (void)sizes; (void)dtypes; (void)fill;\n";
    for (auto& v : scalars)
      if (!std::count(F.params.begin(), F.params.end(), v))
        q << "  " << (floats.count(v) ? T_ : std::string("int64_t")) << " " << cname(v) << " = 0;\n";
    for (auto& [a, ty] : alloc_ty) {
      q << "  int64_t n_" << a << " = 0;\n";
      if (written.count(a)) {
        const std::string et = int_arrays_.count(a) ? "int64_t" : T_;
        q << "  std::vector<" << et << "> v_" << a << ";\n  " << et << "* p_" << a << " = nullptr;\n";
      }
    }
    init_printing_ = true;
    init_stmts(q, F.body, locals, alloc_ty, written, 2, mf_stacks);
    init_printing_ = false;
    q << "  return 0;\n}\n";
    return q.str();
  }

  void init_stmts(std::ostringstream& q, const std::vector<SP>& body, std::set<std::string> locals,
                  const std::map<std::string, std::string>& alloc_ty,
                  const std::set<std::string>& written, int ind, std::string& mf_stacks) {
    const std::string pad(ind, ' ');
    for (auto& sp : body) {
      Stmt& s = *sp;
      switch (s.kind) {
        case Stmt::Assign:
          if (s.lhs->kind == Expr::Var && s.rhs->kind == Expr::Curly) {
            const std::string& a = s.lhs->s;
            q << pad << "n_" << a << " = jl_imax((int64_t)0, (int64_t)("
              << cx(s.rhs->a[1], locals, s.line) << "));\n";
            if (written.count(a))
              q << pad << "v_" << a << ".assign((size_t)n_" << a << ", 0);\n" << pad << "p_" << a
                << " = v_" << a << ".data();\n";
          } else if (s.lhs->kind == Expr::Var) {
            q << pad << cname(s.lhs->s) << " = " << cast_to(s.lhs->s, cx(s.rhs, locals, s.line))
              << ";\n";
          } else {
            // a table write outside the table's size makes the call fail (-1)
            const std::string& a = s.lhs->s;
            q << pad << "{\n" << pad << "  const int64_t o_ = " << offset(s.lhs, locals, s.line)
              << ";\n" << pad << "  if (o_ < 0 || o_ >= n_" << a << ") return -1;\n" << pad
              << "  p_" << a << "[o_] = " << (int_arrays_.count(a) ? "(int64_t)" : "(" + T_ + ")")
              << cx(s.rhs, locals, s.line) << ";\n" << pad << "}\n";
          }
          break;
        case Stmt::For: {
          const std::string v = cname(s.var);
          q << pad << "{\n" << pad << "  const int64_t lo_ = " << cx(s.lo, locals, s.line)
            << ", hi_ = " << cx(s.hi, locals, s.line)
            << ", st_ = " << (s.step ? cx(s.step, locals, s.line) : "((int64_t)1)") << ";\n";
          q << pad << "  for (int64_t " << v << " = lo_; st_ > 0 ? " << v << " <= hi_ : " << v
            << " >= hi_; " << v << " += st_) {\n";
          std::set<std::string> inner = locals;
          inner.insert(s.var);
          init_stmts(q, s.body, inner, alloc_ty, written, ind + 4, mf_stacks);
          q << pad << "  }\n" << pad << "}\n";
          break;
        }
        case Stmt::If:
          q << pad << "if (" << cx(s.cond, locals, s.line) << ") {\n";
          init_stmts(q, s.body, locals, alloc_ty, written, ind + 2, mf_stacks);
          q << pad << "} else {\n";
          init_stmts(q, s.els, locals, alloc_ty, written, ind + 2, mf_stacks);
          q << pad << "}\n";
          break;
        case Stmt::While:
          q << pad << "while (" << cx(s.cond, locals, s.line) << ") {\n";
          init_stmts(q, s.body, locals, alloc_ty, written, ind + 2, mf_stacks);
          q << pad << "}\n";
          break;
        case Stmt::Return: {
          std::vector<EP> items;
          if (s.ret) items = s.ret->kind == Expr::Tuple ? s.ret->a : std::vector<EP>{s.ret};
          std::string ms;
          for (size_t i = 0; i < items.size(); ++i) {
            if (items[i]->kind != Expr::Var) fail(s.line, "initstacks returns " + text(items[i]));
            const std::string& nm = items[i]->s;
            const std::string at = "[" + std::to_string(i) + "]";
            std::string dt;
            auto al = alloc_ty.find(nm);
            if (al == alloc_ty.end()) {
              if (!locals.count(nm) || !ints_.count(nm))
                fail(s.line, "initstacks returns " + nm + ", neither an array it allocates nor an integer");
              q << pad << "if (sizes) sizes" << at << " = " << cname(nm) << ";\n";
              q << pad << "if (dtypes) dtypes" << at << " = 3;\n";
              dt = "int";
            } else {
              const bool is_int = al->second.find("Int") != std::string::npos;
              int code = written.count(nm) ? (is_int ? 4 : 5) : (is_int ? 2 : (f32_ ? 1 : 0));
              q << pad << "if (sizes) sizes" << at << " = n_" << nm << ";\n";
              q << pad << "if (dtypes) dtypes" << at << " = " << code << ";\n";
              if (written.count(nm))
                q << pad << "if (fill && fill" << at << " && n_" << nm << " > 0) memcpy(fill" << at
                  << ", p_" << nm << ", (size_t)n_" << nm << " * sizeof(*p_" << nm << "));\n";
              static const char* names[] = {"f64", "f32", "i64", "int", "i64_table", "float_table"};
              dt = code == 5 ? (f32_ ? "f32_table" : "f64_table") : names[code];
            }
            ms += std::string(ms.empty() ? "" : ", ") + "{\"name\": " + jstr(nm) +
                  ", \"dtype\": " + jstr(dt) + "}";
          }
          mf_stacks = "[" + ms + "]";
          q << pad << "return " << items.size() << ";\n";
          break;
        }
      }
    }
  }

  std::set<std::string> init_locals() {
    std::set<std::string> l;
    if (init_) {
      for (auto& p : init_->params) l.insert(p);
      for (auto& s : init_->body)
        if (s->kind == Stmt::Assign && s->lhs->kind == Expr::Var) l.insert(s->lhs->s);
    }
    return l;
  }

  std::string prelude() {
    return R"PRE(#include <stdint.h>
#include <string.h>
#include <math.h>
#include <vector>
static int64_t stade_launches_ = 0;   // kernels this module has launched
// the grid of a kernel with block sums: at most this many blocks (one slot each)
#define STADE_MAX_RES_BLOCKS 4096
#ifdef STADE_EMIT_HOST
// Host build of the same program (tests): kernels run as loops over their
// threads, in thread order; atomics are plain adds.
struct stade_dim3_ { unsigned x = 0; };
static stade_dim3_ blockIdx, threadIdx, blockDim, gridDim;
#define __global__ static
#define __device__ static
#define __restrict__
typedef void* cudaStream_t;
template <class T, class U> static T atomicAdd(T* p, U v) { T o = *p; *p = (T)(o + (T)v); return o; }
#define STADE_LAUNCH(k, nb, nt, s, ...) do { blockDim.x = (nt); gridDim.x = (nb); ++stade_launches_; \
  for (unsigned b_ = 0; b_ < (unsigned)(nb); ++b_) for (unsigned t_ = 0; t_ < (unsigned)(nt); ++t_) { \
    blockIdx.x = b_; threadIdx.x = t_; k(__VA_ARGS__); } } while (0)
#define STADE_GEN_CHECK() do { } while (0)
#define STADE_CLEAR_ERROR() do { } while (0)
static int stade_box_read(void* dst, const void* box, size_t n, cudaStream_t) { memcpy(dst, box, n); return 0; }
// a thread per iteration, in order, as the sequential loop adds
static int stade_resident_blocks(const void*) { return 1 << 30; }
#define JL_FN(name) static inline double jl_##name(double x) { return name(x); } \
                    static inline float jl_##name(float x) { return name##f(x); }
#else
#include <cuda_runtime.h>
#define STADE_LAUNCH(k, nb, nt, s, ...) do { k<<<(nb), (nt), 0, (s)>>>(__VA_ARGS__); ++stade_launches_; } while (0)
#define STADE_GEN_CHECK() do { if (cudaGetLastError() != cudaSuccess) return 2; } while (0)
#define STADE_CLEAR_ERROR() do { (void)cudaGetLastError(); } while (0)
// blocks of 256 threads the device holds at once for kernel k (a grid-stride
// kernel launched with that many blocks makes one pass)
static int stade_resident_blocks(const void* k) {
  int d = 0, sms = 0, per = 0;
  if (cudaGetDevice(&d) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d) != cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, k, 256, 0) != cudaSuccess || per < 1) {
    (void)cudaGetLastError();
    return 1 << 30;
  }
  return sms * per;
}
template <class B>
static int stade_box_read(void* dst, const B& box, size_t n, cudaStream_t s) {
  if (cudaMemcpyFromSymbolAsync(dst, box, n, 0, cudaMemcpyDeviceToHost, s) != cudaSuccess) return 1;
  return cudaStreamSynchronize(s) == cudaSuccess ? 0 : 1;
}
#define JL_FN(name) __device__ __forceinline__ double jl_##name(double x) { return name(x); } \
                    __device__ __forceinline__ float jl_##name(float x) { return name##f(x); }
// Atomic add aggregated over the lanes of a warp that hit the same address
// (one atomic per address per warp, as the generated __stade_wa_add! does).
template <class T>
__device__ __forceinline__ void jl_atomic_add(T* p, T v) {
  const unsigned mask = __activemask();
  const unsigned lane = threadIdx.x & 31u;
  const unsigned peers = __match_any_sync(mask, (unsigned long long)p);
  if (!__any_sync(mask, __popc(peers) > 1)) {
    atomicAdd(p, v);
    return;
  }
  // every lane of a peer group walks the group's lanes in the same order
  T sum = (T)0;
  for (unsigned m = peers; m; m &= m - 1u) sum += __shfl_sync(peers, v, __ffs(m) - 1);
  if ((unsigned)(__ffs(peers) - 1) == lane) atomicAdd(p, sum);
}
#endif
#ifdef STADE_EMIT_HOST
template <class T> static inline void jl_atomic_add(T* p, T v) { *p = (T)(*p + v); }
template <class T> static inline void jl_block_add(T* p, T v) { *p = (T)(*p + v); }
template <class T> static inline int64_t jl_bits(T) { return 0; }
template <class T> static inline T jl_after(T v, int64_t) { return v; }
#define STADE_ASC 0
#else
// Block sums without float atomics. jl_block_part: the block's sum (warp
// shuffles, then the warps' sums, a fixed tree) into this block's slot;
// jl_block_last: true in the block that finished last (an integer ticket);
// jl_block_finish (that block): the slots summed in block order (each thread
// a contiguous run, then the same fixed tree) and added to the target. With
// the grid fixed (the resident grid of the device), the same sums in the same
// order on every call.
template <class T>
__device__ __forceinline__ T jl_block_reduce(T v) {
  __shared__ T part_[32];
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) part_[w] = v;
  __syncthreads();
  T t = (T)0;
  if (w == 0) {
    t = l < (int)(blockDim.x >> 5) ? part_[l] : (T)0;
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  return t;   // the block's sum in thread 0
}
template <class T>
__device__ __forceinline__ void jl_block_part(T* parts, T v) {
  const T t = jl_block_reduce(v);
  if (threadIdx.x == 0) parts[blockIdx.x] = t;
}
__device__ __forceinline__ bool jl_block_last(unsigned* ticket) {
  __shared__ bool last_;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();   // this block's slots are visible before its ticket
    last_ = atomicAdd(ticket, 1u) == gridDim.x - 1;
  }
  __syncthreads();
  if (last_) __threadfence();
  return last_;
}
template <class T>
__device__ __forceinline__ void jl_block_finish(T* p, const T* parts) {
  const int n = (int)gridDim.x, per = (n + (int)blockDim.x - 1) / (int)blockDim.x;
  const int b0 = (int)threadIdx.x * per, b1 = b0 + per < n ? b0 + per : n;
  T s = (T)0;
  for (int b = b0; b < b1; ++b) s += ((const volatile T*)parts)[b];
  const T t = jl_block_reduce(s);
  if (threadIdx.x == 0) *p += t;
}
// the bits of a loaded value, and v made to depend on them (d is 0 at run time)
__device__ __forceinline__ int64_t jl_bits(double x) { return __double_as_longlong(x); }
__device__ __forceinline__ int64_t jl_bits(float x) { return (int64_t)__float_as_int(x); }
__device__ __forceinline__ int64_t jl_bits(int64_t x) { return x; }
__device__ __forceinline__ double jl_after(double v, int64_t d) {
  return __longlong_as_double(__double_as_longlong(v) | d);
}
__device__ __forceinline__ float jl_after(float v, int64_t d) {
  return __int_as_float(__float_as_int(v) | (int)d);
}
__device__ __forceinline__ int64_t jl_after(int64_t v, int64_t d) { return v | d; }
// threads of a reversed parallel loop take its iterations in ascending address order
#define STADE_ASC 1
#endif
#ifdef STADE_EMIT_HOST
#define JL_HD static inline
#else
#define JL_HD __host__ __device__ __forceinline__
#endif
JL_FN(sqrt) JL_FN(exp) JL_FN(log) JL_FN(tanh) JL_FN(sin) JL_FN(cos) JL_FN(tan) JL_FN(sinh)
JL_FN(cosh) JL_FN(asin) JL_FN(acos) JL_FN(atan) JL_FN(log2) JL_FN(log10) JL_FN(exp2)
JL_FN(expm1) JL_FN(log1p) JL_FN(cbrt)
// Julia's integer division family (div truncates, fld floors, mod takes the divisor's sign)
// 64-bit division is a long instruction sequence on the GPU; index arithmetic
// is almost always non-negative and below 2^31, where 32-bit division gives
// the same quotient.
JL_HD bool jl_small(int64_t a, int64_t b) {
  return (uint64_t)a <= 0x7fffffffull && (uint64_t)(b - 1) < 0x7fffffffull;
}
JL_HD int64_t jl_div(int64_t a, int64_t b) {
  return jl_small(a, b) ? (int64_t)((uint32_t)a / (uint32_t)b) : a / b;
}
JL_HD int64_t jl_rem(int64_t a, int64_t b) {
  return jl_small(a, b) ? (int64_t)((uint32_t)a % (uint32_t)b) : a % b;
}
JL_HD int64_t jl_fld(int64_t a, int64_t b) { int64_t q = a / b; return (q * b != a && ((a < 0) != (b < 0))) ? q - 1 : q; }
JL_HD int64_t jl_cld(int64_t a, int64_t b) { int64_t q = a / b; return (q * b != a && ((a < 0) == (b < 0))) ? q + 1 : q; }
JL_HD int64_t jl_mod(int64_t a, int64_t b) {
  if (jl_small(a, b)) return (int64_t)((uint32_t)a % (uint32_t)b);
  int64_t r = a % b;
  return (r != 0 && ((r < 0) != (b < 0))) ? r + b : r;
}
JL_HD int64_t jl_mod1(int64_t a, int64_t b) { int64_t r = jl_mod(a, b); return r == 0 ? b : r; }
// Division by a divisor d fixed for a kernel (a host integer argument): with
// l = ceil(log2 d) and m = floor(2^32 (2^l - d) / d) + 1, the quotient of
// x < 2^31 is (umulhi(x, m) + x) >> l (Granlund and Montgomery, "Division by
// invariant integers using multiplication", PLDI 1994). m and l are made on
// the host once per launch; outside jl_small's range the plain division runs.
struct jl_fd { uint32_t m, l; };
static inline jl_fd jl_fd_make(int64_t d) {
  jl_fd f{1u, 0u};
  if (d < 1 || d > 0x80000000ll) return f;
  while (((uint64_t)1 << f.l) < (uint64_t)d) ++f.l;
  f.m = (uint32_t)(((((uint64_t)1 << f.l) - (uint64_t)d) << 32) / (uint64_t)d + 1);
  return f;
}
JL_HD uint32_t jl_fd_q(uint32_t x, jl_fd f) {
#ifdef __CUDA_ARCH__
  const uint32_t t = __umulhi(x, f.m);
#else
  const uint32_t t = (uint32_t)(((uint64_t)x * f.m) >> 32);
#endif
  return (t + x) >> f.l;
}
JL_HD int64_t jl_divf(int64_t a, int64_t b, jl_fd f) {
  return jl_small(a, b) ? (int64_t)jl_fd_q((uint32_t)a, f) : a / b;
}
JL_HD int64_t jl_remf(int64_t a, int64_t b, jl_fd f) {
  return jl_small(a, b) ? (int64_t)((uint32_t)a - jl_fd_q((uint32_t)a, f) * (uint32_t)b) : a % b;
}
JL_HD int64_t jl_modf(int64_t a, int64_t b, jl_fd f) {
  return jl_small(a, b) ? jl_remf(a, b, f) : jl_mod(a, b);
}
JL_HD int64_t jl_imax(int64_t a, int64_t b) { return a > b ? a : b; }
JL_HD int64_t jl_imin(int64_t a, int64_t b) { return a < b ? a : b; }
JL_HD int64_t jl_iabs(int64_t a) { return a < 0 ? -a : a; }
JL_HD int64_t jl_isign(int64_t a) { return (a > 0) - (a < 0); }
JL_HD int64_t jl_ipow(int64_t a, int64_t k) { int64_t r = 1; while (k-- > 0) r *= a; return r; }
JL_HD int64_t jl_sq(int64_t a) { return a * a; }
JL_HD int64_t jl_cube(int64_t a) { return a * a * a; }
// Float max / min as Julia's: NaN wins, and max(-0.0, 0.0) = 0.0
template <class T> JL_HD T jl_max(T a, T b) {
  if (a != a) return a; if (b != b) return b;
  if (a == b) return signbit(a) ? b : a;
  return a > b ? a : b;
}
template <class T> JL_HD T jl_min(T a, T b) {
  if (a != a) return a; if (b != b) return b;
  if (a == b) return signbit(a) ? a : b;
  return a < b ? a : b;
}
template <class T> JL_HD T jl_abs(T a) { return a < 0 ? -a : (a == 0 ? (T)0 : a); }
template <class T> JL_HD T jl_sign(T a) { return a > 0 ? (T)1 : (a < 0 ? (T)-1 : a); }
JL_HD double jl_sq(double a) { return a * a; }
JL_HD float jl_sq(float a) { return a * a; }
JL_HD double jl_cube(double a) { return a * a * a; }
JL_HD float jl_cube(float a) { return a * a * a; }
JL_HD double jl_pow(double a, double b) { return pow(a, b); }
JL_HD float jl_pow(float a, float b) { return powf(a, b); }
// trip count of lo:st:hi (0 when empty)
static inline int64_t jl_trip(int64_t lo, int64_t st, int64_t hi) {
  if (st > 0) return hi < lo ? 0 : (hi - lo) / st + 1;
  if (st < 0) return hi > lo ? 0 : (lo - hi) / (-st) + 1;
  return 0;
}
)PRE";
  }
};

std::string g_error;

}  // namespace stade_emit

using namespace stade_emit;

static int emit_impl(const char* source, const char* function, int precision, const char* dims,
                     std::string& cu, std::string& manifest) {
  if (!source) throw Error("source is null");
  if (precision != 64 && precision != 32) throw Error("precision must be 64 or 32");
  Parser p(lex(source));
  std::vector<Func> fs = p.file();
  if (fs.empty()) throw Error("no function in the source");
  Func* f = nullptr;
  if (function && *function) {
    for (auto& x : fs)
      if (x.name == function) f = &x;
    if (!f) throw Error(std::string("no function named ") + function);
  } else {
    for (auto& x : fs) {
      if (x.name.rfind("initstacks_", 0) == 0) continue;
      for (auto& y : fs)
        if (y.name == "initstacks_" + x.name) f = &x;
      if (f) break;
    }
    if (!f)
      for (auto& x : fs)
        if (x.name.rfind("initstacks_", 0) != 0) {
          f = &x;
          break;
        }
    if (!f) throw Error("no sweep function in the source");
  }
  // an HVP sweep <k>_hv takes the stacks of the adjoint's initstacks_<k>_b
  std::string base = f->name;
  if (base.size() > 3 && base.compare(base.size() - 3, 3, "_hv") == 0)
    base = base.substr(0, base.size() - 3) + "_b";
  const Func* init = nullptr;
  for (auto& x : fs)
    if (x.name == "initstacks_" + f->name) init = &x;
  if (!init)
    for (auto& x : fs)
      if (x.name == "initstacks_" + base) init = &x;
  Emitter e(*f, init, precision, dims ? dims : "");
  e.run();
  cu = e.cu;
  manifest = e.manifest;
  return 0;
}

extern "C" int stade_emit_cuda(const char* source, const char* function, int precision,
                               const char* dims, char* cu, size_t cu_cap, size_t* cu_len,
                               char* manifest, size_t manifest_cap, size_t* manifest_len) {
  try {
    std::string c, m;
    emit_impl(source, function, precision, dims, c, m);
    if (cu_len) *cu_len = c.size();
    if (manifest_len) *manifest_len = m.size();
    if (cu && cu_cap > c.size()) std::memcpy(cu, c.c_str(), c.size() + 1);
    if (manifest && manifest_cap > m.size()) std::memcpy(manifest, m.c_str(), m.size() + 1);
    g_error.clear();
    return 0;
  } catch (const std::exception& ex) {
    g_error = ex.what();
    return 1;
  }
}

extern "C" const char* stade_emit_last_error(void) { return g_error.c_str(); }

#ifdef STADE_EMIT_MAIN
// stade_emit in.jl out.cu [--function f] [--precision 32] [--dims "a=m,n"] [--manifest m.json]
#include <fstream>
#include <iostream>
int main(int argc, char** argv) {
  if (argc < 3) {
    std::cerr << "usage: stade_emit in.jl out.cu [--function f] [--precision 64|32] "
                 "[--dims \"a=m,n;b=k\"] [--manifest out.json]\n";
    return 2;
  }
  std::string fn, dims, mpath;
  int prec = 64;
  for (int i = 3; i + 1 < argc; i += 2) {
    std::string k = argv[i];
    if (k == "--function") fn = argv[i + 1];
    else if (k == "--precision") prec = std::atoi(argv[i + 1]);
    else if (k == "--dims") dims = argv[i + 1];
    else if (k == "--manifest") mpath = argv[i + 1];
    else {
      std::cerr << "unknown option " << k << "\n";
      return 2;
    }
  }
  std::ifstream in(argv[1]);
  if (!in) {
    std::cerr << "cannot read " << argv[1] << "\n";
    return 1;
  }
  std::string src((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
  std::string cu, man;
  try {
    emit_impl(src.c_str(), fn.empty() ? nullptr : fn.c_str(), prec, dims.c_str(), cu, man);
  } catch (const std::exception& ex) {
    std::cerr << "stade_emit: " << ex.what() << "\n";
    return 1;
  }
  std::ofstream(argv[2]) << cu;
  if (!mpath.empty()) std::ofstream(mpath) << man;
  return 0;
}
#endif

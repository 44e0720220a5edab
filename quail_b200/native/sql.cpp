// SQL front end: lexer and recursive-descent parser for the query subset the
// engine runs, producing a JSON syntax tree the Python binder plans from.
//
// The reference parses with DataFusion's sqlparser (Snowflake dialect by
// default, BigQuery optional) and registers AI.* as scalar UDFs
// (crates/quail-datafusion/src/functions/mod.rs:42-205). This parser covers
// the statements those queries use: WITH, SELECT [DISTINCT] ... FROM ...
// [JOIN ... ON ...] WHERE ... GROUP BY ... HAVING ... ORDER BY ... LIMIT /
// OFFSET, UNION ALL, EXPLAIN [ANALYZE], SET, and expressions with AND/OR/NOT,
// comparisons, arithmetic, || concatenation, IS [NOT] NULL, [NOT] IN,
// BETWEEN, [NOT] LIKE / ILIKE, CASE, CAST / ::, function calls with dotted
// names (AI.IF, AI.CLASSIFY, PROMPT, HINT, COUNT(*), COUNT(DISTINCT x)),
// array literals ['a', 'b'], Snowflake object literals {'k': v}, BigQuery
// STRUCT(v AS k) and subscripts x['k'] / x[1].
#include <algorithm>
#include <cctype>
#include <stdexcept>
#include <string>
#include <vector>

#include "native.h"

namespace qbn {

namespace {

enum class Tok { Ident, QuotedIdent, Keyword, Number, String, Op, End };

struct Token {
  Tok kind;
  std::string text;  // keywords upper-cased; identifiers as written
  size_t pos;
};

const char* kKeywords[] = {"SELECT", "FROM",   "WHERE",  "GROUP",   "BY",       "HAVING", "ORDER",   "LIMIT",
                           "OFFSET", "AS",     "AND",    "OR",      "NOT",      "IN",     "IS",      "NULL",
                           "TRUE",   "FALSE",  "JOIN",   "INNER",   "LEFT",     "RIGHT",  "FULL",    "OUTER",
                           "CROSS",  "ON",     "USING",  "CASE",    "WHEN",     "THEN",   "ELSE",    "END",
                           "DISTINCT", "ASC",  "DESC",   "BETWEEN", "LIKE",     "ILIKE",  "CAST",    "WITH",
                           "UNION",  "ALL",    "NULLS",  "FIRST",   "LAST",     "EXISTS", "STRUCT",  "QUALIFY",
                           "SET",    "EXPLAIN", "ANALYZE", nullptr};

bool is_keyword(const std::string& up) {
  for (const char** k = kKeywords; *k; ++k)
    if (up == *k) return true;
  return false;
}

std::string upper(std::string s) {
  for (auto& c : s) c = (char)std::toupper((unsigned char)c);
  return s;
}

std::vector<Token> lex(const std::string& src) {
  std::vector<Token> out;
  size_t i = 0;
  const size_t n = src.size();
  while (i < n) {
    const char c = src[i];
    if (std::isspace((unsigned char)c)) {
      ++i;
      continue;
    }
    if (c == '-' && i + 1 < n && src[i + 1] == '-') {
      while (i < n && src[i] != '\n') ++i;
      continue;
    }
    if (c == '/' && i + 1 < n && src[i + 1] == '*') {
      const size_t e = src.find("*/", i + 2);
      if (e == std::string::npos) throw SqlError("unterminated comment", i);
      i = e + 2;
      continue;
    }
    const size_t start = i;
    if (std::isalpha((unsigned char)c) || c == '_') {
      while (i < n && (std::isalnum((unsigned char)src[i]) || src[i] == '_' || src[i] == '$')) ++i;
      std::string word = src.substr(start, i - start);
      std::string up = upper(word);
      if (is_keyword(up))
        out.push_back({Tok::Keyword, up, start});
      else
        out.push_back({Tok::Ident, word, start});
      continue;
    }
    if (c == '"' || c == '`') {
      const char q = c;
      ++i;
      std::string s;
      while (true) {
        if (i >= n) throw SqlError("unterminated quoted identifier", start);
        if (src[i] == q) {
          if (i + 1 < n && src[i + 1] == q) {
            s += q;
            i += 2;
            continue;
          }
          ++i;
          break;
        }
        s += src[i++];
      }
      out.push_back({Tok::QuotedIdent, s, start});
      continue;
    }
    if (c == '\'') {
      ++i;
      std::string s;
      while (true) {
        if (i >= n) throw SqlError("unterminated string literal", start);
        if (src[i] == '\'') {
          if (i + 1 < n && src[i + 1] == '\'') {
            s += '\'';
            i += 2;
            continue;
          }
          ++i;
          break;
        }
        if (src[i] == '\\' && i + 1 < n) {
          const char e = src[i + 1];
          if (e == 'n') s += '\n';
          else if (e == 't') s += '\t';
          else if (e == '\\') s += '\\';
          else if (e == '\'') s += '\'';
          else {
            s += '\\';
            s += e;
          }
          i += 2;
          continue;
        }
        s += src[i++];
      }
      out.push_back({Tok::String, s, start});
      continue;
    }
    if (std::isdigit((unsigned char)c) || (c == '.' && i + 1 < n && std::isdigit((unsigned char)src[i + 1]))) {
      while (i < n && (std::isdigit((unsigned char)src[i]) || src[i] == '.')) ++i;
      if (i < n && (src[i] == 'e' || src[i] == 'E')) {
        ++i;
        if (i < n && (src[i] == '+' || src[i] == '-')) ++i;
        while (i < n && std::isdigit((unsigned char)src[i])) ++i;
      }
      out.push_back({Tok::Number, src.substr(start, i - start), start});
      continue;
    }
    static const char* two[] = {"<=", ">=", "<>", "!=", "||", "::", "=>", nullptr};
    bool matched = false;
    for (const char** t = two; *t; ++t) {
      if (src.compare(i, 2, *t) == 0) {
        out.push_back({Tok::Op, *t, start});
        i += 2;
        matched = true;
        break;
      }
    }
    if (matched) continue;
    if (std::string("=<>+-*/%(),.;[]{}:").find(c) != std::string::npos) {
      out.push_back({Tok::Op, std::string(1, c), start});
      ++i;
      continue;
    }
    throw SqlError(std::string("unexpected character '") + c + "'", i);
  }
  out.push_back({Tok::End, "", n});
  return out;
}

class Parser {
 public:
  explicit Parser(std::vector<Token> toks) : t_(std::move(toks)) {}

  Json statement() {
    Json q;
    if (kw("EXPLAIN")) {
      ++p_;
      const bool analyze = accept_kw("ANALYZE");
      Json inner = query();
      q = node("explain");
      q.set("analyze", analyze);
      q.set("query", inner);
    } else if (kw("SET")) {
      ++p_;
      std::string nm = dotted_name();
      expect_op("=");
      Json value = primary();
      q = node("set");
      q.set("name", nm);
      q.set("value", value);
    } else {
      q = query();
    }
    accept_op(";");
    if (cur().kind != Tok::End) fail("unexpected trailing input");
    return q;
  }

 private:
  std::vector<Token> t_;
  size_t p_ = 0;

  const Token& cur() const { return t_[p_]; }
  const Token& peek(size_t k = 1) const { return t_[std::min(p_ + k, t_.size() - 1)]; }
  [[noreturn]] void fail(const std::string& msg) const {
    throw SqlError(msg + (cur().kind == Tok::End ? " at end of input" : " near '" + cur().text + "'"), cur().pos);
  }
  bool kw(const char* k) const { return cur().kind == Tok::Keyword && cur().text == k; }
  bool op(const char* o) const { return cur().kind == Tok::Op && cur().text == o; }
  bool accept_kw(const char* k) {
    if (kw(k)) {
      ++p_;
      return true;
    }
    return false;
  }
  bool accept_op(const char* o) {
    if (op(o)) {
      ++p_;
      return true;
    }
    return false;
  }
  void expect_kw(const char* k) {
    if (!accept_kw(k)) fail(std::string("expected ") + k);
  }
  void expect_op(const char* o) {
    if (!accept_op(o)) fail(std::string("expected '") + o + "'");
  }
  bool is_name() const { return cur().kind == Tok::Ident || cur().kind == Tok::QuotedIdent; }
  std::string name() {
    if (!is_name()) fail("expected a name");
    return t_[p_++].text;
  }
  std::string dotted_name() {
    std::string s = name();
    while (op(".")) {
      ++p_;
      s += "." + name();
    }
    return s;
  }
  Json node(const char* type) {
    Json j = Json::object();
    j.set("type", type);
    return j;
  }

  // ------------------------------------------------------------ queries
  Json query() {
    Json withs = Json::array();
    if (accept_kw("WITH")) {
      do {
        Json w = Json::object();
        w.set("name", name());
        expect_kw("AS");
        expect_op("(");
        w.set("query", query());
        expect_op(")");
        withs.push(w);
      } while (accept_op(","));
    }
    Json body = set_expr();
    if (withs.size()) body.set("with", withs);
    return body;
  }

  Json set_expr() {
    Json left = select_core();
    while (kw("UNION")) {
      ++p_;
      const bool all = accept_kw("ALL");
      accept_kw("DISTINCT");
      Json right = select_core();
      Json u = node("union");
      u.set("all", all);
      u.set("left", left);
      u.set("right", right);
      left = u;
    }
    if (kw("ORDER")) left.set("order_by", order_by());
    if (accept_kw("LIMIT")) left.set("limit", expr());
    if (accept_kw("OFFSET")) left.set("offset", expr());
    return left;
  }

  Json order_by() {
    expect_kw("ORDER");
    expect_kw("BY");
    Json items = Json::array();
    do {
      Json o = Json::object();
      o.set("expr", expr());
      bool desc = false;
      if (accept_kw("DESC")) desc = true;
      else accept_kw("ASC");
      o.set("desc", desc);
      if (accept_kw("NULLS")) {
        if (accept_kw("FIRST")) {
          o.set("nulls_first", true);
        } else {
          expect_kw("LAST");
          o.set("nulls_first", false);
        }
      }
      items.push(o);
    } while (accept_op(","));
    return items;
  }

  Json select_core() {
    if (op("(")) {
      ++p_;
      Json q = query();
      expect_op(")");
      return q;
    }
    expect_kw("SELECT");
    Json s = node("select");
    s.set("distinct", accept_kw("DISTINCT"));
    Json items = Json::array();
    do {
      Json it = Json::object();
      if (op("*")) {
        ++p_;
        it.set("expr", node("star"));
      } else {
        it.set("expr", expr());
        if (accept_kw("AS")) it.set("alias", name());
        else if (is_name()) it.set("alias", name());
      }
      items.push(it);
    } while (accept_op(","));
    s.set("items", items);
    if (accept_kw("FROM")) {
      Json from = Json::array();
      from.push(table_ref());
      Json joins = Json::array();
      while (true) {
        if (accept_op(",")) {
          Json j = Json::object();
          j.set("kind", "cross");
          j.set("table", table_ref());
          joins.push(j);
          continue;
        }
        std::string kind;
        if (accept_kw("CROSS")) kind = "cross";
        else if (accept_kw("INNER")) kind = "inner";
        else if (accept_kw("LEFT")) { accept_kw("OUTER"); kind = "left"; }
        else if (accept_kw("RIGHT")) { accept_kw("OUTER"); kind = "right"; }
        else if (accept_kw("FULL")) { accept_kw("OUTER"); kind = "full"; }
        else if (kw("JOIN")) kind = "inner";
        else break;
        expect_kw("JOIN");
        Json j = Json::object();
        j.set("kind", kind);
        j.set("table", table_ref());
        if (accept_kw("ON")) {
          j.set("on", expr());
        } else if (accept_kw("USING")) {
          expect_op("(");
          Json cols = Json::array();
          do cols.push(name()); while (accept_op(","));
          expect_op(")");
          j.set("using", cols);
        }
        joins.push(j);
      }
      s.set("from", from);
      if (joins.size()) s.set("joins", joins);
    }
    if (accept_kw("WHERE")) s.set("where", expr());
    if (kw("GROUP")) {
      ++p_;
      expect_kw("BY");
      Json g = Json::array();
      do g.push(expr()); while (accept_op(","));
      s.set("group_by", g);
    }
    if (accept_kw("HAVING")) s.set("having", expr());
    if (accept_kw("QUALIFY")) s.set("qualify", expr());
    return s;
  }

  Json table_ref() {
    Json r = Json::object();
    if (op("(")) {
      ++p_;
      r.set("type", "subquery");
      r.set("query", query());
      expect_op(")");
    } else {
      r.set("type", "table");
      r.set("name", dotted_name());
    }
    if (accept_kw("AS")) r.set("alias", name());
    else if (is_name()) r.set("alias", name());
    return r;
  }

  // ------------------------------------------------------------ expressions
  Json binary(const std::string& o, Json l, Json r) {
    Json j = node("binary");
    j.set("op", o);
    j.set("left", l);
    j.set("right", r);
    return j;
  }

  Json expr() { return or_expr(); }
  Json or_expr() {
    Json l = and_expr();
    while (accept_kw("OR")) l = binary("OR", l, and_expr());
    return l;
  }
  Json and_expr() {
    Json l = not_expr();
    while (accept_kw("AND")) l = binary("AND", l, not_expr());
    return l;
  }
  Json not_expr() {
    if (accept_kw("NOT")) {
      Json j = node("unary");
      j.set("op", "NOT");
      j.set("arg", not_expr());
      return j;
    }
    return predicate();
  }
  Json predicate() {
    Json l = additive();
    while (true) {
      static const char* cmps[] = {"=", "<>", "!=", "<=", ">=", "<", ">", nullptr};
      bool did = false;
      for (const char** c = cmps; *c; ++c) {
        if (op(*c)) {
          ++p_;
          std::string o = *c;
          if (o == "!=") o = "<>";
          l = binary(o, l, additive());
          did = true;
          break;
        }
      }
      if (did) continue;
      if (kw("IS")) {
        ++p_;
        const bool neg = accept_kw("NOT");
        Json j;
        if (accept_kw("NULL")) {
          j = node("is_null");
          j.set("arg", l);
        } else if (kw("TRUE") || kw("FALSE")) {
          const bool val = cur().text == "TRUE";
          ++p_;
          j = node("is_bool");
          j.set("arg", l);
          j.set("value", val);
        } else {
          fail("expected NULL, TRUE or FALSE after IS");
        }
        j.set("negated", neg);
        l = j;
        continue;
      }
      bool neg = false;
      if (kw("NOT") && peek().kind == Tok::Keyword &&
          (peek().text == "IN" || peek().text == "BETWEEN" || peek().text == "LIKE" || peek().text == "ILIKE")) {
        ++p_;
        neg = true;
      }
      if (accept_kw("IN")) {
        expect_op("(");
        Json j = node("in");
        j.set("arg", l);
        if (kw("SELECT") || kw("WITH")) {
          j.set("query", query());
        } else {
          Json items = Json::array();
          do items.push(expr()); while (accept_op(","));
          j.set("list", items);
        }
        expect_op(")");
        j.set("negated", neg);
        l = j;
        continue;
      }
      if (accept_kw("BETWEEN")) {
        Json j = node("between");
        j.set("arg", l);
        j.set("low", additive());
        expect_kw("AND");
        j.set("high", additive());
        j.set("negated", neg);
        l = j;
        continue;
      }
      if (kw("LIKE") || kw("ILIKE")) {
        const bool ci = cur().text == "ILIKE";
        ++p_;
        Json j = node("like");
        j.set("arg", l);
        j.set("pattern", additive());
        j.set("negated", neg);
        j.set("case_insensitive", ci);
        l = j;
        continue;
      }
      if (neg) fail("expected IN, BETWEEN or LIKE after NOT");
      break;
    }
    return l;
  }
  Json additive() {
    Json l = multiplicative();
    while (op("+") || op("-") || op("||")) {
      std::string o = t_[p_++].text;
      l = binary(o, l, multiplicative());
    }
    return l;
  }
  Json multiplicative() {
    Json l = unary();
    while (op("*") || op("/") || op("%")) {
      std::string o = t_[p_++].text;
      l = binary(o, l, unary());
    }
    return l;
  }
  Json unary() {
    if (op("-") || op("+")) {
      std::string o = t_[p_++].text;
      Json a = unary();
      if (o == "+") return a;
      Json j = node("unary");
      j.set("op", "-");
      j.set("arg", a);
      return j;
    }
    return postfix();
  }
  Json postfix() {
    Json e = primary();
    while (true) {
      if (op("::")) {
        ++p_;
        Json j = node("cast");
        j.set("arg", e);
        j.set("to", type_name());
        e = j;
        continue;
      }
      if (op("[")) {
        ++p_;
        Json j = node("subscript");
        j.set("arg", e);
        j.set("index", expr());
        expect_op("]");
        e = j;
        continue;
      }
      break;
    }
    return e;
  }
  std::string type_name() {
    std::string t;
    if (cur().kind == Tok::Ident || cur().kind == Tok::Keyword) t = upper(t_[p_++].text);
    else fail("expected a type name");
    if (accept_op("(")) {
      t += "(";
      while (!op(")")) {
        if (cur().kind == Tok::End) fail("unterminated type");
        t += t_[p_++].text;
      }
      expect_op(")");
      t += ")";
    }
    return t;
  }
  Json literal(const char* kind, Json value) {
    Json j = node("literal");
    j.set("kind", kind);
    j.set("value", value);
    return j;
  }
  Json primary() {
    const Token tk = cur();
    if (tk.kind == Tok::Number) {
      ++p_;
      const bool is_int = tk.text.find_first_of(".eE") == std::string::npos;
      return literal(is_int ? "int" : "float", is_int ? Json(std::stoll(tk.text)) : Json(std::stod(tk.text)));
    }
    if (tk.kind == Tok::String) {
      ++p_;
      return literal("string", Json(tk.text));
    }
    if (accept_kw("NULL")) return literal("null", Json());
    if (accept_kw("TRUE")) return literal("bool", Json(true));
    if (accept_kw("FALSE")) return literal("bool", Json(false));
    if (accept_kw("CASE")) {
      Json j = node("case");
      if (!kw("WHEN")) j.set("operand", expr());
      Json whens = Json::array();
      while (accept_kw("WHEN")) {
        Json w = Json::array();
        w.push(expr());
        expect_kw("THEN");
        w.push(expr());
        whens.push(w);
      }
      if (!whens.size()) fail("CASE needs at least one WHEN");
      j.set("whens", whens);
      if (accept_kw("ELSE")) j.set("else", expr());
      expect_kw("END");
      return j;
    }
    if (accept_kw("CAST")) {
      expect_op("(");
      Json j = node("cast");
      j.set("arg", expr());
      expect_kw("AS");
      j.set("to", type_name());
      expect_op(")");
      return j;
    }
    if (accept_kw("EXISTS")) {
      expect_op("(");
      Json j = node("exists");
      j.set("query", query());
      expect_op(")");
      return j;
    }
    if (accept_kw("STRUCT")) {
      // BigQuery: STRUCT(v AS k, ...)
      expect_op("(");
      Json j = node("object");
      Json items = Json::array();
      if (!op(")")) {
        do {
          Json v = expr();
          expect_kw("AS");
          Json kv = Json::array();
          kv.push(Json(name()));
          kv.push(v);
          items.push(kv);
        } while (accept_op(","));
      }
      expect_op(")");
      j.set("items", items);
      return j;
    }
    if (accept_op("(")) {
      if (kw("SELECT") || kw("WITH")) {
        Json j = node("scalar_subquery");
        j.set("query", query());
        expect_op(")");
        return j;
      }
      Json e = expr();
      expect_op(")");
      return e;
    }
    if (accept_op("[")) {
      Json j = node("array");
      Json items = Json::array();
      if (!op("]")) {
        do items.push(expr()); while (accept_op(","));
      }
      expect_op("]");
      j.set("items", items);
      return j;
    }
    if (accept_op("{")) {
      // Snowflake object literal {'k': v, ...}
      Json j = node("object");
      Json items = Json::array();
      if (!op("}")) {
        do {
          if (cur().kind != Tok::String && !is_name()) fail("expected an object key");
          std::string key = t_[p_++].text;
          expect_op(":");
          Json kv = Json::array();
          kv.push(Json(key));
          kv.push(expr());
          items.push(kv);
        } while (accept_op(","));
      }
      expect_op("}");
      j.set("items", items);
      return j;
    }
    if (is_name() || (tk.kind == Tok::Keyword && (tk.text == "LEFT" || tk.text == "RIGHT"))) {
      // name, dotted name, or function call
      std::vector<std::string> parts;
      parts.push_back(t_[p_++].text);
      while (op(".")) {
        if (peek().kind == Tok::Op && peek().text == "*") {
          p_ += 2;
          Json j = node("star");
          j.set("table", parts.back());
          return j;
        }
        if (peek().kind != Tok::Ident && peek().kind != Tok::QuotedIdent) break;
        ++p_;
        parts.push_back(t_[p_++].text);
      }
      if (op("(")) {
        ++p_;
        std::string fname;
        for (size_t i = 0; i < parts.size(); ++i) fname += (i ? "." : "") + parts[i];
        Json j = node("call");
        j.set("name", upper(fname));
        Json args = Json::array();
        if (accept_kw("DISTINCT")) j.set("distinct", true);
        if (op("*")) {
          ++p_;
          args.push(node("star"));
        } else if (!op(")")) {
          do {
            if (is_name() && peek().kind == Tok::Op && peek().text == "=>") {
              Json na = node("named_arg");
              na.set("name", name());
              ++p_;
              na.set("value", expr());
              args.push(na);
            } else {
              args.push(expr());
            }
          } while (accept_op(","));
        }
        expect_op(")");
        j.set("args", args);
        return j;
      }
      Json j = node("column");
      if (parts.size() == 1) {
        j.set("name", parts[0]);
      } else {
        std::string table;
        for (size_t i = 0; i + 1 < parts.size(); ++i) table += (i ? "." : "") + parts[i];
        j.set("table", table);
        j.set("name", parts.back());
      }
      return j;
    }
    fail("expected an expression");
  }
};

}  // namespace

std::string parse_sql(const std::string& text) {
  Parser p(lex(text));
  return p.statement().dump();
}

}  // namespace qbn

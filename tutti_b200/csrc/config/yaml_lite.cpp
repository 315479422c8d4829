#include "yaml_lite.h"

#include <cctype>
#include <cstdio>
#include <cstdlib>

namespace tutti {
namespace yaml {

namespace {

struct Line {
    int number;
    int indent;
    std::string text;  // without indentation and comments, right-trimmed
};

std::string rtrim(std::string s) {
    while (!s.empty() && std::isspace(static_cast<unsigned char>(s.back()))) s.pop_back();
    return s;
}
std::string trim(const std::string& s) {
    std::size_t a = 0;
    while (a < s.size() && std::isspace(static_cast<unsigned char>(s[a]))) ++a;
    return rtrim(s.substr(a));
}

// Strip a trailing comment that is not inside quotes.
std::string strip_comment(const std::string& s) {
    char q = 0;
    for (std::size_t i = 0; i < s.size(); ++i) {
        const char c = s[i];
        if (q) {
            if (c == q) q = 0;
            continue;
        }
        if (c == '"' || c == '\'') q = c;
        if (c == '#' && (i == 0 || std::isspace(static_cast<unsigned char>(s[i - 1])))) return s.substr(0, i);
    }
    return s;
}

Status err(int line, const std::string& msg) {
    return {StatusCode::INVALID_ARGUMENT, "yaml line " + std::to_string(line) + ": " + msg};
}

NodePtr scalar(const std::string& v, int line) {
    auto n = std::make_shared<Node>();
    n->line = line;
    std::string s = trim(v);
    if (s.empty() || s == "~" || s == "null") {
        n->kind = Node::Kind::Null;
        return n;
    }
    n->kind = Node::Kind::Scalar;
    if (s.size() >= 2 && ((s.front() == '"' && s.back() == '"') || (s.front() == '\'' && s.back() == '\''))) {
        std::string out;
        const bool dq = s.front() == '"';
        for (std::size_t i = 1; i + 1 < s.size(); ++i) {
            if (dq && s[i] == '\\' && i + 2 < s.size()) {
                const char e = s[++i];
                out += e == 'n' ? '\n' : e == 't' ? '\t' : e;
            } else if (!dq && s[i] == '\'' && i + 2 < s.size() && s[i + 1] == '\'') {
                out += '\'';
                ++i;
            } else {
                out += s[i];
            }
        }
        n->scalar = out;
    } else {
        n->scalar = s;
    }
    return n;
}

// ---- flow collections -------------------------------------------------------
struct Flow {
    const std::string& s;
    std::size_t i = 0;
    int line;
    void ws() {
        while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
    }
    Result<NodePtr> value() {
        ws();
        if (i >= s.size()) return Result<NodePtr>::Failure(err(line, "unexpected end of flow collection"));
        if (s[i] == '{') return map();
        if (s[i] == '[') return seq();
        return plain();
    }
    Result<NodePtr> plain() {
        ws();
        std::size_t a = i;
        if (i < s.size() && (s[i] == '"' || s[i] == '\'')) {
            const char q = s[i++];
            while (i < s.size() && s[i] != q) ++i;
            if (i >= s.size()) return Result<NodePtr>::Failure(err(line, "unterminated quote"));
            ++i;
            return scalar(s.substr(a, i - a), line);
        }
        while (i < s.size() && s[i] != ',' && s[i] != ']' && s[i] != '}' && s[i] != ':') ++i;
        return scalar(s.substr(a, i - a), line);
    }
    Result<NodePtr> seq() {
        auto n = std::make_shared<Node>();
        n->kind = Node::Kind::Seq;
        n->line = line;
        ++i;  // [
        ws();
        if (i < s.size() && s[i] == ']') {
            ++i;
            return n;
        }
        for (;;) {
            auto v = value();
            if (!v.ok()) return v;
            n->seq.push_back(v.value());
            ws();
            if (i < s.size() && s[i] == ',') {
                ++i;
                continue;
            }
            if (i < s.size() && s[i] == ']') {
                ++i;
                return n;
            }
            return Result<NodePtr>::Failure(err(line, "expected ',' or ']' in flow sequence"));
        }
    }
    Result<NodePtr> map() {
        auto n = std::make_shared<Node>();
        n->kind = Node::Kind::Map;
        n->line = line;
        ++i;  // {
        ws();
        if (i < s.size() && s[i] == '}') {
            ++i;
            return n;
        }
        for (;;) {
            auto k = plain();
            if (!k.ok()) return k;
            ws();
            if (i >= s.size() || s[i] != ':') return Result<NodePtr>::Failure(err(line, "expected ':' in flow mapping"));
            ++i;
            auto v = value();
            if (!v.ok()) return v;
            n->map.emplace_back(k.value()->scalar, v.value());
            ws();
            if (i < s.size() && s[i] == ',') {
                ++i;
                continue;
            }
            if (i < s.size() && s[i] == '}') {
                ++i;
                return n;
            }
            return Result<NodePtr>::Failure(err(line, "expected ',' or '}' in flow mapping"));
        }
    }
};

Result<NodePtr> inline_value(const std::string& v, int line) {
    const std::string t = trim(v);
    if (!t.empty() && (t[0] == '{' || t[0] == '[')) {
        Flow f{t, 0, line};
        auto r = f.value();
        if (!r.ok()) return r;
        f.ws();
        if (f.i != t.size()) return Result<NodePtr>::Failure(err(line, "trailing characters after flow collection"));
        return r;
    }
    if (!t.empty() && (t[0] == '&' || t[0] == '*' || t[0] == '!' || t[0] == '|' || t[0] == '>'))
        return Result<NodePtr>::Failure(err(line, "anchors, aliases, tags and block scalars are not supported"));
    return scalar(t, line);
}

// Position of the key/value ':' separator outside quotes, or npos.
std::size_t key_colon(const std::string& s) {
    char q = 0;
    for (std::size_t i = 0; i < s.size(); ++i) {
        const char c = s[i];
        if (q) {
            if (c == q) q = 0;
            continue;
        }
        if (c == '"' || c == '\'') q = c;
        if (c == '{' || c == '[') return std::string::npos;
        if (c == ':' && (i + 1 == s.size() || s[i + 1] == ' ')) return i;
    }
    return std::string::npos;
}

struct Parser {
    std::vector<Line> lines;
    std::size_t pos = 0;

    Result<NodePtr> block(int indent) {
        if (pos >= lines.size()) return scalar("", lines.empty() ? 0 : lines.back().number);
        const Line& first = lines[pos];
        if (first.indent < indent) return scalar("", first.number);
        if (first.text.rfind("- ", 0) == 0 || first.text == "-") return sequence(first.indent);
        return mapping(first.indent);
    }

    Result<NodePtr> mapping(int indent) {
        auto n = std::make_shared<Node>();
        n->kind = Node::Kind::Map;
        n->line = lines[pos].number;
        while (pos < lines.size() && lines[pos].indent == indent) {
            const Line& l = lines[pos];
            if (l.text.rfind("- ", 0) == 0) break;
            const std::size_t c = key_colon(l.text);
            if (c == std::string::npos) return Result<NodePtr>::Failure(err(l.number, "expected 'key: value'"));
            auto key = scalar(l.text.substr(0, c), l.number);
            const std::string rest = trim(l.text.substr(c + 1));
            for (auto& kv : n->map)
                if (kv.first == key->scalar) return Result<NodePtr>::Failure(err(l.number, "duplicate key '" + key->scalar + "'"));
            ++pos;
            if (!rest.empty()) {
                auto v = inline_value(rest, l.number);
                if (!v.ok()) return v;
                n->map.emplace_back(key->scalar, v.value());
            } else if (pos < lines.size() && (lines[pos].indent > indent ||
                                              (lines[pos].indent == indent && lines[pos].text.rfind("- ", 0) == 0))) {
                auto v = block(lines[pos].indent);
                if (!v.ok()) return v;
                n->map.emplace_back(key->scalar, v.value());
            } else {
                n->map.emplace_back(key->scalar, scalar("", l.number));
            }
        }
        if (pos < lines.size() && lines[pos].indent > indent)
            return Result<NodePtr>::Failure(err(lines[pos].number, "unexpected indentation"));
        return n;
    }

    Result<NodePtr> sequence(int indent) {
        auto n = std::make_shared<Node>();
        n->kind = Node::Kind::Seq;
        n->line = lines[pos].number;
        while (pos < lines.size() && lines[pos].indent == indent &&
               (lines[pos].text.rfind("- ", 0) == 0 || lines[pos].text == "-")) {
            Line l = lines[pos];
            const std::string rest = l.text.size() > 1 ? trim(l.text.substr(2)) : "";
            if (rest.empty()) {
                ++pos;
                auto v = block(pos < lines.size() ? lines[pos].indent : indent + 2);
                if (!v.ok()) return v;
                n->seq.push_back(v.value());
                continue;
            }
            if (key_colon(rest) != std::string::npos) {
                // "- key: value" opens a mapping whose keys sit at indent + 2
                lines[pos].indent = indent + 2;
                lines[pos].text = rest;
                auto v = mapping(indent + 2);
                if (!v.ok()) return v;
                n->seq.push_back(v.value());
                continue;
            }
            ++pos;
            auto v = inline_value(rest, l.number);
            if (!v.ok()) return v;
            n->seq.push_back(v.value());
        }
        return n;
    }
};

}  // namespace

const Node* Node::get(const std::string& key) const {
    for (auto& kv : map)
        if (kv.first == key) return kv.second.get();
    return nullptr;
}

Result<NodePtr> parse(const std::string& text) {
    Parser p;
    int number = 0;
    std::size_t a = 0;
    while (a <= text.size()) {
        std::size_t b = text.find('\n', a);
        if (b == std::string::npos) b = text.size();
        std::string raw = text.substr(a, b - a);
        ++number;
        a = b + 1;
        if (raw.find('\t') != std::string::npos && raw.find_first_not_of(" \t") != std::string::npos &&
            raw.find('\t') < raw.find_first_not_of(" \t"))
            return Result<NodePtr>::Failure(err(number, "tabs are not allowed for indentation"));
        std::string s = rtrim(strip_comment(raw));
        if (trim(s).empty()) {
            if (b == text.size()) break;
            continue;
        }
        if (trim(s) == "---") continue;
        if (trim(s) == "...") break;
        int indent = 0;
        while (indent < static_cast<int>(s.size()) && s[indent] == ' ') ++indent;
        p.lines.push_back({number, indent, s.substr(indent)});
        if (b == text.size()) break;
    }
    if (p.lines.empty()) return scalar("", 0);
    auto r = p.block(p.lines[0].indent);
    if (!r.ok()) return r;
    if (p.pos != p.lines.size()) return Result<NodePtr>::Failure(err(p.lines[p.pos].number, "unexpected content"));
    return r;
}

Result<NodePtr> parse_file(const std::string& path) {
    std::FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) return Result<NodePtr>::Failure({StatusCode::NOT_FOUND, "cannot open " + path});
    std::string text;
    char buf[4096];
    std::size_t n;
    while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) text.append(buf, n);
    std::fclose(f);
    return parse(text);
}

Result<std::int64_t> as_int(const Node& n, const std::string& path) {
    if (!n.is_scalar()) return Result<std::int64_t>::Failure(err(n.line, path + ": expected an integer"));
    char* end = nullptr;
    const long long v = std::strtoll(n.scalar.c_str(), &end, 0);
    if (!end || *end != '\0' || n.scalar.empty())
        return Result<std::int64_t>::Failure(err(n.line, path + ": '" + n.scalar + "' is not an integer"));
    return static_cast<std::int64_t>(v);
}

Result<bool> as_bool(const Node& n, const std::string& path) {
    if (n.is_scalar()) {
        if (n.scalar == "true" || n.scalar == "True" || n.scalar == "yes") return true;
        if (n.scalar == "false" || n.scalar == "False" || n.scalar == "no") return false;
    }
    return Result<bool>::Failure(err(n.line, path + ": expected true or false"));
}

Result<std::string> as_string(const Node& n, const std::string& path) {
    if (!n.is_scalar()) return Result<std::string>::Failure(err(n.line, path + ": expected a string"));
    return n.scalar;
}

}  // namespace yaml
}  // namespace tutti

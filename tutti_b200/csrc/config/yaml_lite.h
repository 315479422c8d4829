#pragma once
// A YAML subset parser for runtime and daemon configuration files.
//
// Supported: block mappings and block sequences by indentation, flow mappings
// `{a: 1, b: [x, y]}` and flow sequences, plain / single- / double-quoted
// scalars, `#` comments, a leading `---`. Not supported (rejected with an
// error): anchors/aliases, tags, multi-line scalars, multiple documents.
// Every node remembers its line so configuration errors can name it.

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include <tutti/status.h>

namespace tutti {
namespace yaml {

struct Node {
    enum class Kind { Null, Scalar, Map, Seq };
    Kind kind = Kind::Null;
    std::string scalar;
    std::vector<std::pair<std::string, std::shared_ptr<Node>>> map;  // insertion order
    std::vector<std::shared_ptr<Node>> seq;
    int line = 0;

    bool is_map() const { return kind == Kind::Map; }
    bool is_seq() const { return kind == Kind::Seq; }
    bool is_scalar() const { return kind == Kind::Scalar; }
    const Node* get(const std::string& key) const;
};

using NodePtr = std::shared_ptr<Node>;

Result<NodePtr> parse(const std::string& text);
Result<NodePtr> parse_file(const std::string& path);

// Scalar conversions; fail with the node's line on mismatch.
Result<std::int64_t> as_int(const Node& n, const std::string& path);
Result<bool> as_bool(const Node& n, const std::string& path);
Result<std::string> as_string(const Node& n, const std::string& path);

}  // namespace yaml
}  // namespace tutti

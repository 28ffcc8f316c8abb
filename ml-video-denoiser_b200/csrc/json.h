// Minimal JSON reader for manifest.json (objects, arrays, strings, numbers,
// booleans, null). Throws dnb::JsonError with a byte offset on malformed input.
#pragma once

#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

namespace dnb {

struct JsonError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    bool b = false;
    double num = 0.0;
    std::string str;
    std::vector<Json> arr;
    std::map<std::string, Json> obj;

    bool has(const std::string& k) const { return kind == Object && obj.count(k) > 0; }
    const Json& at(const std::string& k) const;
    std::string get_string(const std::string& k, const std::string& def) const;
    long long get_int(const std::string& k, long long def) const;
    bool get_bool(const std::string& k, bool def) const;
};

Json parse_json(const std::string& text);

}  // namespace dnb

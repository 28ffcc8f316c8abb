#include "json.h"

#include <cctype>
#include <cstdlib>

namespace dnb {
namespace {

struct Parser {
    const std::string& s;
    size_t i = 0;

    [[noreturn]] void fail(const char* what) const {
        throw JsonError(std::string("manifest JSON: ") + what + " at byte " + std::to_string(i));
    }
    void ws() {
        while (i < s.size() && std::isspace(static_cast<unsigned char>(s[i]))) ++i;
    }
    bool eat(char c) {
        ws();
        if (i < s.size() && s[i] == c) {
            ++i;
            return true;
        }
        return false;
    }
    void expect(char c) {
        if (!eat(c)) fail((std::string("expected '") + c + "'").c_str());
    }

    std::string parse_string() {
        ws();
        if (i >= s.size() || s[i] != '"') fail("expected string");
        ++i;
        std::string out;
        while (i < s.size() && s[i] != '"') {
            char c = s[i++];
            if (c == '\\') {
                if (i >= s.size()) fail("bad escape");
                const char e = s[i++];
                switch (e) {
                    case '"': out += '"'; break;
                    case '\\': out += '\\'; break;
                    case '/': out += '/'; break;
                    case 'b': out += '\b'; break;
                    case 'f': out += '\f'; break;
                    case 'n': out += '\n'; break;
                    case 'r': out += '\r'; break;
                    case 't': out += '\t'; break;
                    case 'u': {
                        if (i + 4 > s.size()) fail("bad \\u escape");
                        const unsigned cp = std::strtoul(s.substr(i, 4).c_str(), nullptr, 16);
                        i += 4;
                        if (cp < 0x80) {
                            out += static_cast<char>(cp);
                        } else if (cp < 0x800) {
                            out += static_cast<char>(0xC0 | (cp >> 6));
                            out += static_cast<char>(0x80 | (cp & 0x3F));
                        } else {
                            out += static_cast<char>(0xE0 | (cp >> 12));
                            out += static_cast<char>(0x80 | ((cp >> 6) & 0x3F));
                            out += static_cast<char>(0x80 | (cp & 0x3F));
                        }
                        break;
                    }
                    default: fail("bad escape");
                }
            } else {
                out += c;
            }
        }
        if (i >= s.size()) fail("unterminated string");
        ++i;
        return out;
    }

    Json parse_value(int depth) {
        if (depth > 64) fail("nesting too deep");
        ws();
        if (i >= s.size()) fail("unexpected end");
        Json v;
        const char c = s[i];
        if (c == '{') {
            ++i;
            v.kind = Json::Object;
            if (eat('}')) return v;
            do {
                std::string k = parse_string();
                expect(':');
                v.obj[k] = parse_value(depth + 1);
            } while (eat(','));
            expect('}');
        } else if (c == '[') {
            ++i;
            v.kind = Json::Array;
            if (eat(']')) return v;
            do {
                v.arr.push_back(parse_value(depth + 1));
            } while (eat(','));
            expect(']');
        } else if (c == '"') {
            v.kind = Json::String;
            v.str = parse_string();
        } else if (s.compare(i, 4, "true") == 0) {
            i += 4;
            v.kind = Json::Bool;
            v.b = true;
        } else if (s.compare(i, 5, "false") == 0) {
            i += 5;
            v.kind = Json::Bool;
        } else if (s.compare(i, 4, "null") == 0) {
            i += 4;
        } else if (c == '-' || std::isdigit(static_cast<unsigned char>(c))) {
            const char* start = s.c_str() + i;
            char* end = nullptr;
            v.num = std::strtod(start, &end);
            if (end == start) fail("bad number");
            i += static_cast<size_t>(end - start);
            v.kind = Json::Number;
        } else {
            fail("unexpected character");
        }
        return v;
    }
};

}  // namespace

const Json& Json::at(const std::string& k) const {
    auto it = obj.find(k);
    if (kind != Object || it == obj.end()) throw JsonError("manifest JSON: missing key '" + k + "'");
    return it->second;
}

std::string Json::get_string(const std::string& k, const std::string& def) const {
    if (!has(k)) return def;
    const Json& v = at(k);
    if (v.kind != String) throw JsonError("manifest JSON: '" + k + "' is not a string");
    return v.str;
}

long long Json::get_int(const std::string& k, long long def) const {
    if (!has(k)) return def;
    const Json& v = at(k);
    if (v.kind != Number) throw JsonError("manifest JSON: '" + k + "' is not a number");
    return static_cast<long long>(v.num);
}

bool Json::get_bool(const std::string& k, bool def) const {
    if (!has(k)) return def;
    const Json& v = at(k);
    if (v.kind != Bool) throw JsonError("manifest JSON: '" + k + "' is not a boolean");
    return v.b;
}

Json parse_json(const std::string& text) {
    Parser p{text};
    Json v = p.parse_value(0);
    p.ws();
    if (p.i != text.size()) p.fail("trailing characters");
    return v;
}

}  // namespace dnb

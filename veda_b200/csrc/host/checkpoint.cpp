// Safetensors writer and reader (include/veda/checkpoint.hpp).
#include "veda/checkpoint.hpp"

#include <cstring>
#include <fstream>
#include <set>
#include <stdexcept>

namespace veda::io
{

namespace
{
[[noreturn]] void fail(const std::string& path, const std::string& why)
{
    throw std::runtime_error("safetensors " + path + ": " + why);
}

std::string json_string(const std::string& s)
{
    std::string out = "\"";
    for (const char c : s)
    {
        switch (c)
        {
        case '"': out += "\\\""; break;
        case '\\': out += "\\\\"; break;
        case '\n': out += "\\n"; break;
        case '\t': out += "\\t"; break;
        default:
            if (static_cast<unsigned char>(c) < 0x20)
            {
                char buf[8];
                std::snprintf(buf, sizeof(buf), "\\u%04x", static_cast<unsigned>(c));
                out += buf;
            }
            else
            {
                out += c;
            }
        }
    }
    return out + "\"";
}

// ---- a JSON reader for the header: objects, arrays, strings, non-negative integers -----------
struct Json
{
    enum Kind { Object, Array, String, Number } kind = Object;
    std::vector<std::pair<std::string, Json>> members;   // Object, in order
    std::vector<Json> items;                             // Array
    std::string text;                                    // String
    uint64_t number = 0;                                 // Number
};

class Parser
{
public:
    explicit Parser(const std::string& s) : s_(s) {}

    Json document()
    {
        Json j = value();
        skip();
        if (at_ != s_.size()) throw std::runtime_error("trailing characters");
        return j;
    }

private:
    void skip()
    {
        while (at_ < s_.size() && (s_[at_] == ' ' || s_[at_] == '\n' || s_[at_] == '\t' || s_[at_] == '\r'))
            ++at_;
    }
    char peek()
    {
        skip();
        if (at_ >= s_.size()) throw std::runtime_error("unexpected end");
        return s_[at_];
    }
    void expect(char c)
    {
        if (peek() != c) throw std::runtime_error(std::string("expected '") + c + "'");
        ++at_;
    }
    Json value()
    {
        const char c = peek();
        if (c == '{') return object();
        if (c == '[') return array();
        if (c == '"')
        {
            Json j;
            j.kind = Json::String;
            j.text = string();
            return j;
        }
        if (c >= '0' && c <= '9') return number();
        throw std::runtime_error(std::string("unsupported value starting with '") + c + "'");
    }
    Json object()
    {
        Json j;
        j.kind = Json::Object;
        expect('{');
        if (peek() == '}')
        {
            ++at_;
            return j;
        }
        for (;;)
        {
            if (peek() != '"') throw std::runtime_error("expected a member name");
            std::string key = string();
            expect(':');
            j.members.emplace_back(std::move(key), value());
            if (peek() == ',')
            {
                ++at_;
                continue;
            }
            expect('}');
            return j;
        }
    }
    Json array()
    {
        Json j;
        j.kind = Json::Array;
        expect('[');
        if (peek() == ']')
        {
            ++at_;
            return j;
        }
        for (;;)
        {
            j.items.push_back(value());
            if (peek() == ',')
            {
                ++at_;
                continue;
            }
            expect(']');
            return j;
        }
    }
    Json number()
    {
        Json j;
        j.kind = Json::Number;
        skip();
        const size_t start = at_;
        while (at_ < s_.size() && s_[at_] >= '0' && s_[at_] <= '9')
        {
            if (j.number > (UINT64_MAX - 9) / 10) throw std::runtime_error("integer too large");
            j.number = j.number * 10 + static_cast<uint64_t>(s_[at_] - '0');
            ++at_;
        }
        if (at_ == start) throw std::runtime_error("expected a digit");
        return j;
    }
    std::string string()
    {
        expect('"');
        std::string out;
        while (at_ < s_.size() && s_[at_] != '"')
        {
            char c = s_[at_++];
            if (c == '\\')
            {
                if (at_ >= s_.size()) break;
                const char e = s_[at_++];
                switch (e)
                {
                case '"': out += '"'; break;
                case '\\': out += '\\'; break;
                case '/': out += '/'; break;
                case 'n': out += '\n'; break;
                case 't': out += '\t'; break;
                case 'r': out += '\r'; break;
                case 'b': out += '\b'; break;
                case 'f': out += '\f'; break;
                case 'u':
                {
                    if (at_ + 4 > s_.size()) throw std::runtime_error("short \\u escape");
                    const unsigned v = static_cast<unsigned>(std::stoul(s_.substr(at_, 4), nullptr, 16));
                    at_ += 4;
                    if (v >= 0x80) throw std::runtime_error("non-ASCII \\u escape");
                    out += static_cast<char>(v);
                    break;
                }
                default: throw std::runtime_error("bad escape");
                }
            }
            else
            {
                out += c;
            }
        }
        if (at_ >= s_.size()) throw std::runtime_error("unterminated string");
        ++at_;
        return out;
    }

    const std::string& s_;
    size_t at_ = 0;
};
} // namespace

size_t dtype_bytes(const std::string& dtype)
{
    if (dtype == "F64" || dtype == "I64" || dtype == "U64") return 8;
    if (dtype == "F32" || dtype == "I32" || dtype == "U32") return 4;
    if (dtype == "BF16" || dtype == "F16" || dtype == "I16" || dtype == "U16") return 2;
    if (dtype == "I8" || dtype == "U8" || dtype == "BOOL") return 1;
    throw std::invalid_argument("safetensors: unknown dtype " + dtype);
}

const SafetensorsTensor& SafetensorsFile::at(const std::string& name) const
{
    for (const auto& t : tensors)
    {
        if (t.name == name) return t;
    }
    throw std::runtime_error("safetensors: no tensor named " + name);
}

void write_safetensors(const std::string& path, const std::vector<SafetensorsTensor>& tensors,
                       const std::map<std::string, std::string>& metadata)
{
    std::string header = "{";
    bool first = true;
    if (!metadata.empty())
    {
        header += "\"__metadata__\":{";
        bool f2 = true;
        for (const auto& [k, v] : metadata)
        {
            header += (f2 ? "" : ",") + json_string(k) + ":" + json_string(v);
            f2 = false;
        }
        header += "}";
        first = false;
    }
    std::set<std::string> seen;
    uint64_t offset = 0;
    for (const auto& t : tensors)
    {
        if (t.name == "__metadata__" || !seen.insert(t.name).second)
        {
            throw std::invalid_argument("safetensors: tensor name " + t.name + " repeats or is reserved");
        }
        uint64_t count = 1;
        for (const int64_t d : t.shape)
        {
            if (d < 0) throw std::invalid_argument("safetensors: negative dimension in " + t.name);
            count *= static_cast<uint64_t>(d);
        }
        if (count * dtype_bytes(t.dtype) != t.bytes.size())
        {
            throw std::invalid_argument("safetensors: " + t.name + " holds " + std::to_string(t.bytes.size()) +
                                        " bytes, its dtype and shape need " +
                                        std::to_string(count * dtype_bytes(t.dtype)));
        }
        header += (first ? "" : ",") + json_string(t.name) + ":{\"dtype\":" + json_string(t.dtype) +
                  ",\"shape\":[";
        for (size_t i = 0; i < t.shape.size(); ++i)
        {
            header += (i ? "," : "") + std::to_string(t.shape[i]);
        }
        header += "],\"data_offsets\":[" + std::to_string(offset) + "," +
                  std::to_string(offset + t.bytes.size()) + "]}";
        offset += t.bytes.size();
        first = false;
    }
    header += "}";
    while (header.size() % 8 != 0)
    {
        header += ' ';
    }
    std::ofstream out(path, std::ios::binary | std::ios::trunc);
    if (!out)
    {
        fail(path, "cannot be opened for writing");
    }
    uint8_t len[8];
    const uint64_t n = header.size();
    for (int i = 0; i < 8; ++i)
    {
        len[i] = static_cast<uint8_t>(n >> (8 * i));
    }
    out.write(reinterpret_cast<const char*>(len), 8);
    out.write(header.data(), static_cast<std::streamsize>(header.size()));
    for (const auto& t : tensors)
    {
        out.write(reinterpret_cast<const char*>(t.bytes.data()), static_cast<std::streamsize>(t.bytes.size()));
    }
    out.flush();
    if (!out)
    {
        fail(path, "write failed");
    }
}

SafetensorsFile read_safetensors(const std::string& path)
{
    std::ifstream in(path, std::ios::binary | std::ios::ate);
    if (!in)
    {
        fail(path, "cannot be opened");
    }
    const uint64_t size = static_cast<uint64_t>(in.tellg());
    if (size < 8)
    {
        fail(path, "is too small to hold a header length");
    }
    in.seekg(0);
    uint8_t len[8];
    in.read(reinterpret_cast<char*>(len), 8);
    uint64_t n = 0;
    for (int i = 0; i < 8; ++i)
    {
        n |= static_cast<uint64_t>(len[i]) << (8 * i);
    }
    if (n > size - 8)
    {
        fail(path, "header length " + std::to_string(n) + " runs past the file");
    }
    std::string header(static_cast<size_t>(n), '\0');
    in.read(header.data(), static_cast<std::streamsize>(n));
    Json doc;
    try
    {
        doc = Parser(header).document();
    }
    catch (const std::exception& e)
    {
        fail(path, std::string("header is not valid JSON: ") + e.what());
    }
    if (doc.kind != Json::Object)
    {
        fail(path, "header is not a JSON object");
    }
    const uint64_t data_start = 8 + n, data_size = size - data_start;
    SafetensorsFile file;
    for (const auto& [name, entry] : doc.members)
    {
        if (name == "__metadata__")
        {
            for (const auto& [k, v] : entry.members)
            {
                if (v.kind == Json::String) file.metadata[k] = v.text;
            }
            continue;
        }
        const Json *dtype = nullptr, *shape = nullptr, *offsets = nullptr;
        for (const auto& [k, v] : entry.members)
        {
            if (k == "dtype") dtype = &v;
            if (k == "shape") shape = &v;
            if (k == "data_offsets") offsets = &v;
        }
        if (!dtype || !shape || !offsets || dtype->kind != Json::String || shape->kind != Json::Array ||
            offsets->kind != Json::Array || offsets->items.size() != 2)
        {
            fail(path, "tensor " + name + ": entry is missing dtype, shape or data_offsets");
        }
        SafetensorsTensor t;
        t.name = name;
        t.dtype = dtype->text;
        uint64_t count = 1;
        for (const Json& d : shape->items)
        {
            t.shape.push_back(static_cast<int64_t>(d.number));
            count *= d.number;
        }
        const uint64_t b = offsets->items[0].number, e = offsets->items[1].number;
        if (e < b || e > data_size || e - b != count * dtype_bytes(t.dtype))
        {
            fail(path, "tensor " + name + ": byte range [" + std::to_string(b) + ", " + std::to_string(e) +
                           ") disagrees with its shape or the data section");
        }
        t.bytes.resize(static_cast<size_t>(e - b));
        in.seekg(static_cast<std::streamoff>(data_start + b));
        in.read(reinterpret_cast<char*>(t.bytes.data()), static_cast<std::streamsize>(e - b));
        if (!in)
        {
            fail(path, "tensor " + name + ": read failed");
        }
        file.tensors.push_back(std::move(t));
    }
    return file;
}

} // namespace veda::io

// The safetensors header parser (a small JSON subset: objects, arrays, strings with escapes, integers, and the
// literals true/false/null) and the tensor reader.
#include "safetensors.hpp"

#include <cstring>
#include <fstream>
#include <stdexcept>

namespace h3 {
namespace {

struct Json {
    enum Kind { Null, Bool, Number, String, Array, Object } kind = Null;
    double num = 0;
    bool b = false;
    std::string str;
    std::vector<Json> arr;
    std::vector<std::pair<std::string, Json>> obj;
};

class Parser {
public:
    explicit Parser(const std::string& s) : s_(s) {}
    Json parse()
    {
        Json v = value();
        ws();
        if (i_ != s_.size())
            fail("trailing characters");
        return v;
    }

private:
    const std::string& s_;
    size_t i_ = 0;

    [[noreturn]] void fail(const char* what) const
    {
        throw std::runtime_error(std::string("safetensors header: ") + what + " at byte " + std::to_string(i_));
    }
    void ws()
    {
        while (i_ < s_.size() && (s_[i_] == ' ' || s_[i_] == '\n' || s_[i_] == '\r' || s_[i_] == '\t'))
            ++i_;
    }
    char peek()
    {
        ws();
        if (i_ >= s_.size())
            fail("unexpected end");
        return s_[i_];
    }
    void expect(char c)
    {
        if (peek() != c)
            fail("unexpected character");
        ++i_;
    }
    std::string string_lit()
    {
        expect('"');
        std::string out;
        while (true) {
            if (i_ >= s_.size())
                fail("unterminated string");
            const char c = s_[i_++];
            if (c == '"')
                return out;
            if (c != '\\') {
                out.push_back(c);
                continue;
            }
            if (i_ >= s_.size())
                fail("unterminated escape");
            const char e = s_[i_++];
            switch (e) {
            case '"': out.push_back('"'); break;
            case '\\': out.push_back('\\'); break;
            case '/': out.push_back('/'); break;
            case 'b': out.push_back('\b'); break;
            case 'f': out.push_back('\f'); break;
            case 'n': out.push_back('\n'); break;
            case 'r': out.push_back('\r'); break;
            case 't': out.push_back('\t'); break;
            case 'u': {
                if (i_ + 4 > s_.size())
                    fail("short \\u escape");
                const unsigned cp = unsigned(std::stoul(s_.substr(i_, 4), nullptr, 16));
                i_ += 4;
                // UTF-8 for the basic plane (the names here are ASCII; anything else is kept readable)
                if (cp < 0x80)
                    out.push_back(char(cp));
                else if (cp < 0x800) {
                    out.push_back(char(0xC0 | (cp >> 6)));
                    out.push_back(char(0x80 | (cp & 0x3F)));
                } else {
                    out.push_back(char(0xE0 | (cp >> 12)));
                    out.push_back(char(0x80 | ((cp >> 6) & 0x3F)));
                    out.push_back(char(0x80 | (cp & 0x3F)));
                }
                break;
            }
            default: fail("bad escape");
            }
        }
    }
    Json value()
    {
        Json v;
        const char c = peek();
        if (c == '{') {
            ++i_;
            v.kind = Json::Object;
            if (peek() == '}') {
                ++i_;
                return v;
            }
            while (true) {
                std::string k = string_lit();
                expect(':');
                v.obj.emplace_back(std::move(k), value());
                const char d = peek();
                ++i_;
                if (d == '}')
                    return v;
                if (d != ',')
                    fail("expected , or }");
            }
        }
        if (c == '[') {
            ++i_;
            v.kind = Json::Array;
            if (peek() == ']') {
                ++i_;
                return v;
            }
            while (true) {
                v.arr.push_back(value());
                const char d = peek();
                ++i_;
                if (d == ']')
                    return v;
                if (d != ',')
                    fail("expected , or ]");
            }
        }
        if (c == '"') {
            v.kind = Json::String;
            v.str = string_lit();
            return v;
        }
        if (s_.compare(i_, 4, "true") == 0 || s_.compare(i_, 5, "false") == 0) {
            v.kind = Json::Bool;
            v.b = s_[i_] == 't';
            i_ += v.b ? 4 : 5;
            return v;
        }
        if (s_.compare(i_, 4, "null") == 0) {
            i_ += 4;
            return v;
        }
        size_t used = 0;
        try {
            v.num = std::stod(s_.substr(i_, 32), &used);
        } catch (const std::exception&) {
            fail("bad number");
        }
        i_ += used;
        v.kind = Json::Number;
        return v;
    }
};

float half_to_float(uint16_t h)
{
    const uint32_t sign = uint32_t(h >> 15) << 31, exp = (h >> 10) & 0x1F, man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0)
            bits = sign;
        else { // subnormal: renormalise
            int e = -1;
            uint32_t m = man;
            do {
                ++e;
                m <<= 1;
            } while (!(m & 0x400));
            bits = sign | uint32_t(127 - 15 - e) << 23 | (m & 0x3FF) << 13;
        }
    } else if (exp == 31)
        bits = sign | 0x7F800000u | man << 13;
    else
        bits = sign | (exp - 15 + 127) << 23 | man << 13;
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

} // namespace

SafeTensors::SafeTensors(const std::string& path) : path_(path)
{
    std::ifstream f(path, std::ios::binary);
    if (!f)
        throw std::runtime_error("safetensors: cannot open " + path);
    unsigned char len8[8];
    if (!f.read(reinterpret_cast<char*>(len8), 8))
        throw std::runtime_error("safetensors: " + path + " is shorter than its header length");
    uint64_t n = 0;
    for (int i = 7; i >= 0; --i)
        n = n << 8 | len8[i];
    if (n == 0 || n > (uint64_t(1) << 30))
        throw std::runtime_error("safetensors: " + path + ": implausible header length " + std::to_string(n));
    std::string header(n, '\0');
    if (!f.read(header.data(), std::streamsize(n)))
        throw std::runtime_error("safetensors: " + path + ": truncated header");
    data_offset_ = 8 + n;
    f.seekg(0, std::ios::end);
    const uint64_t file_size = uint64_t(f.tellg());
    const Json root = Parser(header).parse();
    if (root.kind != Json::Object)
        throw std::runtime_error("safetensors: " + path + ": the header is not an object");
    for (const auto& [name, v] : root.obj) {
        if (name == "__metadata__") {
            for (const auto& [k, mv] : v.obj)
                if (mv.kind == Json::String)
                    meta_[k] = mv.str;
            continue;
        }
        SafeTensor t;
        for (const auto& [k, fv] : v.obj) {
            if (k == "dtype")
                t.dtype = fv.str;
            else if (k == "shape")
                for (const Json& d : fv.arr)
                    t.shape.push_back(int64_t(d.num));
            else if (k == "data_offsets" && fv.arr.size() == 2)
                t.begin = uint64_t(fv.arr[0].num), t.end = uint64_t(fv.arr[1].num);
        }
        if (t.end < t.begin || data_offset_ + t.end > file_size)
            throw std::runtime_error("safetensors: " + path + ": tensor " + name + " lies outside the file");
        tensors_[name] = std::move(t);
    }
}

std::vector<unsigned char> SafeTensors::read_raw(const std::string& name, const SafeTensor*& tp) const
{
    const auto it = tensors_.find(name);
    if (it == tensors_.end())
        throw std::runtime_error("safetensors: " + path_ + " has no tensor " + name);
    const SafeTensor& t = it->second;
    tp = &t;
    uint64_t count = 1;
    for (int64_t d : t.shape)
        count *= uint64_t(d);
    const uint64_t esz = t.dtype == "F32" ? 4 : (t.dtype == "BF16" || t.dtype == "F16") ? 2 : 0;
    if (!esz)
        throw std::runtime_error("safetensors: tensor " + name + " has dtype " + t.dtype + " (BF16, F16 or F32 expected)");
    if (count * esz != t.end - t.begin)
        throw std::runtime_error("safetensors: tensor " + name + ": its shape and byte range disagree");
    std::vector<unsigned char> raw(t.end - t.begin);
    std::ifstream f(path_, std::ios::binary);
    f.seekg(std::streamoff(data_offset_ + t.begin));
    if (!f.read(reinterpret_cast<char*>(raw.data()), std::streamsize(raw.size())))
        throw std::runtime_error("safetensors: " + path_ + ": cannot read tensor " + name);
    return raw;
}

uint16_t bf16_bits(float f)
{
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x007FFFFFu))
        return uint16_t((u >> 16) | 0x40); // NaN stays a (quiet) NaN
    u += 0x7FFFu + ((u >> 16) & 1u);
    return uint16_t(u >> 16);
}

std::vector<uint16_t> SafeTensors::read_bf16(const std::string& name) const
{
    const SafeTensor* t = nullptr;
    const std::vector<unsigned char> raw = read_raw(name, t);
    if (t->dtype == "BF16") {
        std::vector<uint16_t> out(raw.size() / 2);
        std::memcpy(out.data(), raw.data(), raw.size());
        return out;
    }
    const std::vector<float> f = read_f32(name);
    std::vector<uint16_t> out(f.size());
    for (size_t i = 0; i < f.size(); ++i)
        out[i] = bf16_bits(f[i]);
    return out;
}

void write_safetensors(const std::string& path, const std::vector<SafeTensorOut>& tensors,
                       const std::map<std::string, std::string>& metadata,
                       const std::function<void(size_t, std::vector<unsigned char>&)>& data)
{
    auto quote = [](const std::string& v) {
        std::string q = "\"";
        for (char ch : v) {
            if (ch == '"' || ch == '\\')
                q += '\\';
            q += ch;
        }
        return q + "\"";
    };
    std::string h = "{";
    if (!metadata.empty()) {
        h += "\"__metadata__\":{";
        bool first = true;
        for (const auto& [k, v] : metadata) {
            h += (first ? "" : ",") + quote(k) + ":" + quote(v);
            first = false;
        }
        h += "}";
    }
    uint64_t off = 0;
    for (size_t i = 0; i < tensors.size(); ++i) {
        const SafeTensorOut& t = tensors[i];
        h += (i || !metadata.empty() ? "," : "") + quote(t.name) + ":{\"dtype\":" + quote(t.dtype) + ",\"shape\":[";
        for (size_t k = 0; k < t.shape.size(); ++k)
            h += (k ? "," : "") + std::to_string(t.shape[k]);
        h += "],\"data_offsets\":[" + std::to_string(off) + "," + std::to_string(off + t.bytes) + "]}";
        off += t.bytes;
    }
    h += "}";
    while (h.size() % 8)
        h += ' ';
    std::ofstream f(path, std::ios::binary | std::ios::trunc);
    if (!f)
        throw std::runtime_error("safetensors: cannot create " + path);
    unsigned char len8[8];
    uint64_t n = h.size();
    for (int i = 0; i < 8; ++i, n >>= 8)
        len8[i] = static_cast<unsigned char>(n & 0xFF);
    f.write(reinterpret_cast<const char*>(len8), 8);
    f.write(h.data(), std::streamsize(h.size()));
    std::vector<unsigned char> buf;
    for (size_t i = 0; i < tensors.size(); ++i) {
        buf.assign(tensors[i].bytes, 0);
        data(i, buf);
        f.write(reinterpret_cast<const char*>(buf.data()), std::streamsize(buf.size()));
    }
    if (!f)
        throw std::runtime_error("safetensors: writing " + path + " failed");
}

std::vector<float> SafeTensors::read_f32(const std::string& name) const
{
    const SafeTensor* tp = nullptr;
    const std::vector<unsigned char> raw = read_raw(name, tp);
    const SafeTensor& t = *tp;
    const uint64_t esz = t.dtype == "F32" ? 4 : 2;
    const uint64_t count = raw.size() / esz;
    std::vector<float> out(count);
    for (uint64_t i = 0; i < count; ++i) {
        if (esz == 4)
            std::memcpy(&out[i], &raw[4 * i], 4);
        else {
            const uint16_t h = uint16_t(raw[2 * i] | raw[2 * i + 1] << 8);
            if (t.dtype == "BF16") {
                const uint32_t bits = uint32_t(h) << 16;
                std::memcpy(&out[i], &bits, 4);
            } else
                out[i] = half_to_float(h);
        }
    }
    return out;
}

} // namespace h3

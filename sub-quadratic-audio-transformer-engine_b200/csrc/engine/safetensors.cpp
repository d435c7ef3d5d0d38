// Safetensors loader: 8-byte little-endian header length, a JSON header of
// {name: {dtype, shape, data_offsets}}, then the raw bytes. Every length and
// offset is checked against the file size before use (the reference checks
// the same bounds, src/safetensors.cpp:84-128); tensors are copied into the
// arena. A small JSON reader covers the header grammar.
#include "safetensors.hpp"

#include <cuda_runtime.h>

#include <climits>
#include <cstdint>
#include <cstring>
#include <fstream>
#include <iterator>
#include <map>
#include <memory>
#include <stdexcept>

namespace {

struct JVal {
    enum Kind { NUL, BOOL, NUM, STR, ARR, OBJ } kind = NUL;
    bool b = false;
    bool integral = false;
    unsigned long long u = 0;  // when integral and non-negative
    double num = 0;
    std::string s;
    std::vector<JVal> arr;
    std::vector<std::pair<std::string, JVal>> obj;
};

class JReader {
public:
    explicit JReader(const std::string& t) : t_(t) {}
    JVal parse_document() {
        JVal v = value(0);
        ws();
        if (i_ != t_.size()) throw std::runtime_error("trailing characters in header");
        return v;
    }

private:
    const std::string& t_;
    size_t i_ = 0;
    void ws() {
        while (i_ < t_.size() && (t_[i_] == ' ' || t_[i_] == '\n' || t_[i_] == '\r' || t_[i_] == '\t')) ++i_;
    }
    char peek() {
        ws();
        if (i_ >= t_.size()) throw std::runtime_error("unexpected end of header");
        return t_[i_];
    }
    void expect(char c) {
        if (peek() != c) throw std::runtime_error(std::string("expected '") + c + "'");
        ++i_;
    }
    JVal value(int depth) {
        if (depth > 32) throw std::runtime_error("header nesting too deep");
        const char c = peek();
        JVal v;
        if (c == '{') {
            ++i_;
            v.kind = JVal::OBJ;
            if (peek() == '}') { ++i_; return v; }
            for (;;) {
                std::string k = str();
                expect(':');
                v.obj.emplace_back(std::move(k), value(depth + 1));
                if (peek() == ',') { ++i_; continue; }
                expect('}');
                return v;
            }
        }
        if (c == '[') {
            ++i_;
            v.kind = JVal::ARR;
            if (peek() == ']') { ++i_; return v; }
            for (;;) {
                v.arr.push_back(value(depth + 1));
                if (peek() == ',') { ++i_; continue; }
                expect(']');
                return v;
            }
        }
        if (c == '"') { v.kind = JVal::STR; v.s = str(); return v; }
        if (t_.compare(i_, 4, "true") == 0) { i_ += 4; v.kind = JVal::BOOL; v.b = true; return v; }
        if (t_.compare(i_, 5, "false") == 0) { i_ += 5; v.kind = JVal::BOOL; return v; }
        if (t_.compare(i_, 4, "null") == 0) { i_ += 4; return v; }
        return number();
    }
    std::string str() {
        expect('"');
        std::string out;
        while (i_ < t_.size() && t_[i_] != '"') {
            if (t_[i_] == '\\') {
                if (++i_ >= t_.size()) break;
                const char e = t_[i_];
                if (e == 'u') { out += '?'; i_ += 4; }
                else out += (e == 'n' ? '\n' : e == 't' ? '\t' : e);
                ++i_;
                continue;
            }
            out += t_[i_++];
        }
        if (i_ >= t_.size()) throw std::runtime_error("unterminated string in header");
        ++i_;
        return out;
    }
    JVal number() {
        const size_t start = i_;
        bool neg = false;
        if (t_[i_] == '-') { neg = true; ++i_; }
        bool integral = true;
        unsigned long long u = 0;
        bool overflow = false;
        size_t digits = 0;
        while (i_ < t_.size() && t_[i_] >= '0' && t_[i_] <= '9') {
            const unsigned d = (unsigned)(t_[i_] - '0');
            if (u > (ULLONG_MAX - d) / 10) overflow = true;
            else u = u * 10 + d;
            ++i_;
            ++digits;
        }
        while (i_ < t_.size() && (t_[i_] == '.' || t_[i_] == 'e' || t_[i_] == 'E' || t_[i_] == '+' || t_[i_] == '-' ||
                                  (t_[i_] >= '0' && t_[i_] <= '9'))) {
            integral = false;
            ++i_;
        }
        if (digits == 0) throw std::runtime_error("malformed number in header");
        JVal v;
        v.kind = JVal::NUM;
        v.num = std::stod(t_.substr(start, i_ - start));
        v.integral = integral && !neg && !overflow;
        v.u = u;
        return v;
    }
};

std::vector<size_t> uint_list(const JVal& v, const char* what) {
    if (v.kind != JVal::ARR) throw std::runtime_error(std::string(what) + " must be a list");
    std::vector<size_t> out;
    for (const JVal& x : v.arr) {
        if (x.kind != JVal::NUM || !x.integral) throw std::runtime_error(std::string(what) + " entries must be unsigned integers");
        out.push_back((size_t)x.u);
    }
    return out;
}

size_t dtype_bytes(const std::string& dt) {
    static const std::map<std::string, size_t> sizes = {
        {"F64", 8}, {"F32", 4}, {"F16", 2}, {"BF16", 2}, {"I64", 8}, {"I32", 4}, {"I16", 2},
        {"I8", 1},  {"U8", 1},  {"BOOL", 1}, {"U16", 2}, {"U32", 4}, {"U64", 8}};
    auto it = sizes.find(dt);
    return it == sizes.end() ? 0 : it->second;
}

}  // namespace

bool SafetensorLoader::load(const std::string& filepath) {
    try {
        std::ifstream f(filepath, std::ios::binary);
        if (!f) return false;
        std::vector<char> bytes((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
        const size_t file_size = bytes.size();
        if (file_size < 8) return false;
        uint64_t header_size = 0;
        std::memcpy(&header_size, bytes.data(), 8);
        if (header_size > file_size - 8) return false;
        const size_t data_start = 8 + (size_t)header_size;
        const std::string header(bytes.data() + 8, (size_t)header_size);
        JVal root = JReader(header).parse_document();
        if (root.kind != JVal::OBJ) return false;
        for (const auto& kv : root.obj) {
            if (kv.first == "__metadata__") continue;
            const JVal& t = kv.second;
            if (t.kind != JVal::OBJ) return false;
            std::string dtype = "F32";
            std::vector<size_t> shape, offsets;
            bool have_shape = false, have_off = false;
            for (const auto& f2 : t.obj) {
                if (f2.first == "dtype" && f2.second.kind == JVal::STR) dtype = f2.second.s;
                else if (f2.first == "shape") { shape = uint_list(f2.second, "shape"); have_shape = true; }
                else if (f2.first == "data_offsets") { offsets = uint_list(f2.second, "data_offsets"); have_off = true; }
            }
            if (!have_shape || !have_off || shape.size() > 4) return false;
            if (offsets.size() != 2 || offsets[0] > offsets[1]) return false;
            if (offsets[1] > file_size || data_start > file_size - offsets[1]) return false;
            const size_t esz = dtype_bytes(dtype);
            if (esz == 0) return false;
            size_t count = 1;
            for (size_t s : shape) {
                if (s != 0 && count > SIZE_MAX / s) return false;
                count *= s;
            }
            if (count > SIZE_MAX / esz || count * esz != offsets[1] - offsets[0]) return false;
            const size_t nbytes = offsets[1] - offsets[0];
            void* dst = arena_.allocate(nbytes);
            if (nbytes && cudaMemcpy(dst, bytes.data() + data_start + offsets[0], nbytes, cudaMemcpyHostToDevice) != cudaSuccess)
                return false;
            SafetensorMetadata m{dtype, shape, offsets[0], offsets[1]};
            meta_[kv.first] = m;
            TensorDescriptor td;
            td.dimensions = shape;
            td.strides.assign(shape.size(), 1);
            for (int i = (int)shape.size() - 2; i >= 0; --i) td.strides[i] = td.strides[i + 1] * shape[i + 1];
            td.precision = dtype == "F16" ? PrecisionMode::FP16 : dtype == "BF16" ? PrecisionMode::BF16 : PrecisionMode::FP32;
            td.data = dst;
            td.is_on_host = false;
            tensors_[kv.first] = td;
        }
        return true;
    } catch (const std::exception&) {
        return false;
    }
}

TensorDescriptor SafetensorLoader::get_tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw std::runtime_error("Tensor '" + name + "' not found in SafetensorLoader.");
    return it->second;
}

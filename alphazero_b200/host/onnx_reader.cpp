#include "onnx_reader.h"

#include <cstring>
#include <fstream>
#include <stdexcept>

namespace mgb {
namespace {

// Protobuf wire-format cursor over [pos, end).  Every read checks bounds.
struct Wire {
    const uint8_t* pos;
    const uint8_t* end;

    bool more() const { return pos < end; }

    uint64_t varint() {
        uint64_t v = 0;
        for (int shift = 0; shift < 64; shift += 7) {
            if (pos >= end) throw std::runtime_error("onnx: truncated varint");
            uint8_t b = *pos++;
            v |= (uint64_t)(b & 0x7f) << shift;
            if (!(b & 0x80)) return v;
        }
        throw std::runtime_error("onnx: varint too long");
    }

    uint32_t fixed32() {
        if (end - pos < 4) throw std::runtime_error("onnx: truncated fixed32");
        uint32_t v;
        std::memcpy(&v, pos, 4);
        pos += 4;
        return v;
    }

    Wire bytes() {
        uint64_t len = varint();
        if (len > (uint64_t)(end - pos)) throw std::runtime_error("onnx: truncated field");
        Wire sub{pos, pos + len};
        pos += len;
        return sub;
    }

    void skip(int wire_type) {
        switch (wire_type) {
            case 0: varint(); break;
            case 1:
                if (end - pos < 8) throw std::runtime_error("onnx: truncated fixed64");
                pos += 8;
                break;
            case 2: bytes(); break;
            case 5: fixed32(); break;
            default: throw std::runtime_error("onnx: unknown wire type");
        }
    }
};

float bits_to_float(uint32_t b) {
    float f;
    std::memcpy(&f, &b, 4);
    return f;
}

NamedTensor parse_tensor(Wire w) {
    NamedTensor t;
    while (w.more()) {
        uint64_t key = w.varint();
        int field = (int)(key >> 3), wt = (int)(key & 7);
        if (field == 1) {
            if (wt == 2) {
                Wire p = w.bytes();
                while (p.more()) t.dims.push_back((int64_t)p.varint());
            } else if (wt == 0) {
                t.dims.push_back((int64_t)w.varint());
            } else {
                w.skip(wt);
            }
        } else if (field == 2 && wt == 0) {
            t.data_type = (int)w.varint();
        } else if (field == 4) {
            if (wt == 2) {
                Wire p = w.bytes();
                while (p.more()) t.float_data.push_back(bits_to_float(p.fixed32()));
            } else if (wt == 5) {
                t.float_data.push_back(bits_to_float(w.fixed32()));
            } else {
                w.skip(wt);
            }
        } else if (field == 8 && wt == 2) {
            Wire s = w.bytes();
            t.name.assign((const char*)s.pos, (size_t)(s.end - s.pos));
        } else if (field == 9 && wt == 2) {
            Wire s = w.bytes();
            t.raw_data.assign(s.pos, s.end);
        } else {
            w.skip(wt);
        }
    }
    return t;
}

std::vector<NamedTensor> parse_graph(Wire w) {
    std::vector<NamedTensor> out;
    while (w.more()) {
        uint64_t key = w.varint();
        int field = (int)(key >> 3), wt = (int)(key & 7);
        if (field == 5 && wt == 2) out.push_back(parse_tensor(w.bytes()));
        else w.skip(wt);
    }
    return out;
}

}  // namespace

int64_t NamedTensor::elements() const {
    if (dims.empty()) return 0;
    int64_t n = 1;
    for (int64_t d : dims) n *= d;
    return n;
}

std::vector<float> NamedTensor::floats() const {
    if (data_type != 0 && data_type != 1)
        throw std::runtime_error("onnx: tensor " + name + " is not FLOAT (data_type " +
                                 std::to_string(data_type) + ")");
    if (!float_data.empty()) return float_data;
    std::vector<float> v(raw_data.size() / 4);
    if (!v.empty()) std::memcpy(v.data(), raw_data.data(), v.size() * 4);
    return v;
}

std::vector<NamedTensor> parse_onnx_initializers(const uint8_t* data, size_t size) {
    Wire w{data, data + size};
    std::vector<NamedTensor> inits;
    while (w.more()) {
        uint64_t key = w.varint();
        int field = (int)(key >> 3), wt = (int)(key & 7);
        if (field == 7 && wt == 2) inits = parse_graph(w.bytes());
        else w.skip(wt);
    }
    return inits;
}

std::vector<NamedTensor> read_onnx_initializers(const std::string& path) {
    std::ifstream f(path, std::ios::binary | std::ios::ate);
    if (!f.is_open()) throw std::runtime_error("Cannot open model file: " + path);
    std::streamsize n = f.tellg();
    f.seekg(0);
    std::vector<uint8_t> buf((size_t)n);
    if (n > 0 && !f.read(reinterpret_cast<char*>(buf.data()), n))
        throw std::runtime_error("Cannot read model file: " + path);
    return parse_onnx_initializers(buf.data(), buf.size());
}

}  // namespace mgb

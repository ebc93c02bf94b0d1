// A minimal safetensors reader and writer (the format the reference's weights and LoRAs ship in): an 8-byte
// little-endian header length, a JSON header {name: {dtype, shape, data_offsets}, "__metadata__": {key: string}},
// then the raw little-endian tensor bytes. The tensor table, the metadata, and a tensor's values as fp32 or bf16
// (BF16, F16 and F32 sources); files of BF16 and F32 tensors are written.
#pragma once

#include <cstdint>
#include <functional>
#include <map>
#include <string>
#include <vector>

namespace h3 {

struct SafeTensor {
    std::string dtype;          // "BF16", "F16", "F32", ...
    std::vector<int64_t> shape;
    uint64_t begin = 0, end = 0; // byte range inside the data section
};

class SafeTensors {
public:
    // Reads the header of `path`; throws std::runtime_error on a malformed file.
    explicit SafeTensors(const std::string& path);
    const std::map<std::string, SafeTensor>& tensors() const { return tensors_; }
    const std::map<std::string, std::string>& metadata() const { return meta_; }
    // The tensor's values converted to fp32 (row-major, as stored).
    std::vector<float> read_f32(const std::string& name) const;
    // The tensor's values as bf16 bit patterns: BF16 as stored, F32 and F16 rounded to the nearest even.
    std::vector<uint16_t> read_bf16(const std::string& name) const;
    const std::string& path() const { return path_; }

private:
    std::vector<unsigned char> read_raw(const std::string& name, const SafeTensor*& t) const;
    std::string path_;
    uint64_t data_offset_ = 0;
    std::map<std::string, SafeTensor> tensors_;
    std::map<std::string, std::string> meta_;
};

// One tensor of a file to write: its name, dtype ("BF16" or "F32"), shape and byte count.
struct SafeTensorOut {
    std::string name, dtype;
    std::vector<int64_t> shape;
    uint64_t bytes = 0;
};

// Writes a safetensors file: the header for `tensors` (their data in this order, the header padded with spaces to a
// multiple of 8 bytes), then each tensor's bytes as `data(i, buffer)` fills them (the buffer sized to the tensor).
void write_safetensors(const std::string& path, const std::vector<SafeTensorOut>& tensors,
                       const std::map<std::string, std::string>& metadata,
                       const std::function<void(size_t, std::vector<unsigned char>&)>& data);

// fp32 to bf16 bits, rounded to the nearest even (NaN kept a NaN).
uint16_t bf16_bits(float f);

} // namespace h3

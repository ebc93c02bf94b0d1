// A minimal safetensors reader (the format the reference's weights and LoRAs ship in): an 8-byte little-endian
// header length, a JSON header {name: {dtype, shape, data_offsets}, "__metadata__": {key: string}}, then the raw
// little-endian tensor bytes. Only what the LoRA merge needs: the tensor table, the metadata, and a tensor's values
// as fp32 (BF16, F16 and F32 sources).
#pragma once

#include <cstdint>
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

private:
    std::string path_;
    uint64_t data_offset_ = 0;
    std::map<std::string, SafeTensor> tensors_;
    std::map<std::string, std::string> meta_;
};

} // namespace h3

// Safetensors files: the writer the reference lacks (it only reads them,
// src/libs/io/Safetensors.cpp:106-257) and a reader for files this writer made.
//
// Layout (the format the reference's reader accepts): an 8-byte little-endian header length N,
// N bytes of JSON — {"__metadata__": {string: string}, name: {"dtype", "shape", "data_offsets"}}
// in the order the tensors were given, padded with spaces to a multiple of 8 bytes — then the
// tensors' raw little-endian bytes back to back, each at its data_offsets relative to the start
// of the data section.
#pragma once

#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace veda::io
{

struct SafetensorsTensor
{
    std::string name;
    std::string dtype;            // "BF16", "F32", "I64", ...
    std::vector<int64_t> shape;
    std::vector<uint8_t> bytes;   // raw little-endian data
};

struct SafetensorsFile
{
    std::map<std::string, std::string> metadata;
    std::vector<SafetensorsTensor> tensors;   // header order
    const SafetensorsTensor& at(const std::string& name) const;   // throws std::runtime_error
};

// Bytes per element of a safetensors dtype name; std::invalid_argument for an unknown one.
size_t dtype_bytes(const std::string& dtype);

// Writes the tensors in the given order. std::invalid_argument if a tensor's byte count does not
// match its dtype and shape or a name repeats; std::runtime_error naming the path on I/O errors.
void write_safetensors(const std::string& path, const std::vector<SafetensorsTensor>& tensors,
                       const std::map<std::string, std::string>& metadata = {});

// Reads a file in the layout above (the JSON subset of objects, arrays, strings and integers).
// std::runtime_error naming the path for a short file, a header past the end, malformed JSON or a
// byte range that disagrees with the shape.
SafetensorsFile read_safetensors(const std::string& path);

} // namespace veda::io

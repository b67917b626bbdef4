// Header reader for the safetensors format (src/formats/safetensors.rs):
// 8-byte little-endian header length, that many bytes of UTF-8 JSON mapping
// tensor names to {"dtype", "shape", "data_offsets"} (plus an ignored
// "__metadata__" entry), then the data.  Host code only: the device loader
// streams the payload a tensor names without widening it on the host.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace krt {

enum StDtype { ST_F32 = 0, ST_BF16 = 1, ST_F16 = 2 };

struct StTensor {
    int dtype;                     // StDtype
    std::vector<uint64_t> shape;
    uint64_t start, end;           // byte range in the data section
};

struct StHeader {
    uint64_t data_offset;          // file offset of the data section (8 + header length)
    uint64_t data_len;             // bytes in the data section
    std::map<std::string, StTensor> tensors;
};

// Validates a header image the way read_with does (safetensors.rs:161-257):
// `prefix` holds the file's first bytes (at least the 8-byte length and, when
// the file has them, the header), `file_len` the whole file's size.  Every
// entry is checked (dtype, shape, offsets against the data section), in the
// key order of the reference's JSON map.  Returns "" or the reference's error
// text (SafeTensorsError's Display, safetensors.rs:46-68).
std::string st_parse(const unsigned char *prefix, size_t prefix_len, uint64_t file_len, StHeader *out);

// st_parse on a file: reads the length, then the header bytes.
std::string st_read_header(const char *path, StHeader *out);

}  // namespace krt

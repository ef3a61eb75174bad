// safetensors.cuh — reader of the safetensors container (host code).
//
// The reference reads MLX checkpoints with the `safetensors` crate
// (SafeTensors::deserialize in load_weights_from_manifest,
// crates/serve/src/loader/weights.rs:43-60; the crate is a dependency, not
// vendored).  This is a restatement of that container's published format:
//   [u64 little-endian n][n bytes of JSON header][data]
// where the header is one JSON object mapping each tensor name to
// {"dtype": "BF16"|"U32"|..., "shape": [d0, d1, ...], "data_offsets": [b, e]}
// (byte range [b, e) of the data section) plus an optional "__metadata__"
// object of strings.  Validation follows the crate's: the header fits the
// file, every tensor's byte count is prod(shape) * dtype size, and the
// tensors tile the data section contiguously from 0 to its end.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace emx {

struct StTensor {
  std::string name;
  std::string dtype;           // as written in the header ("BF16", "U32", ...)
  std::vector<int64_t> shape;
  uint64_t offset = 0;         // byte offset of the data in the file
  uint64_t bytes = 0;
};

// A read-only mapping of one .safetensors file and its tensors (header order).
struct StFile {
  std::string path;
  const unsigned char* base = nullptr;  // the whole file, mapped
  size_t size = 0;
  std::vector<StTensor> tensors;
  StFile() = default;
  StFile(const StFile&) = delete;
  StFile& operator=(const StFile&) = delete;
  ~StFile();
};

// Bytes per element of a safetensors dtype name, or 0 when unknown.
int st_dtype_size(const std::string& dtype);

// Maps and validates `path`.  Returns EMX_OK or EMX_ERR_INVALID (message set).
int st_open(const char* path, StFile* out);

// Parses a header (no mapping): the same validation against a data section
// of `data_bytes` bytes.  Used by st_open and by tests of malformed headers.
int st_parse_header(const char* json, size_t len, uint64_t data_bytes, uint64_t data_start,
                    std::vector<StTensor>* out, const char* what);

// The "weight_map" of a model.safetensors.index.json: the distinct shard file
// names in first-seen order.
int st_index_files(const char* index_path, std::vector<std::string>* files);

}  // namespace emx

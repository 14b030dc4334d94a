// Safetensors checkpoint files (the MLX 4-bit checkpoints the reference loads,
// full_forward.swift:451-472, 555-595, 749-822): each file is an 8-byte
// little-endian header length, a JSON header mapping tensor names to
// {"dtype", "shape", "data_offsets": [begin, end]} (offsets relative to the
// end of the header) plus an optional "__metadata__" object, then the data.
// Files are memory-mapped read-only; tensor data is read in place.
#pragma once
#include <cstddef>
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace iam {

struct StTensor {
  std::string name;   // as stored in the file
  std::string dtype;  // "U32", "BF16", "F32", ...
  std::vector<int64_t> shape;
  uint64_t begin = 0, end = 0;  // byte range in the file's data section
  int file = 0;
  size_t bytes() const { return static_cast<size_t>(end - begin); }
};

struct StFile {
  std::string path;
  const unsigned char* base = nullptr;  // the whole file, mapped
  size_t size = 0;
  size_t data_off = 0;  // 8 + header length
};

struct StCheckpoint {
  std::vector<StFile> files;
  std::map<std::string, StTensor> tensors;  // by the engine's name (see st_engine_name)
  std::vector<std::string> ignored;         // names with no engine counterpart form (other towers, ...)
  ~StCheckpoint();
  const void* data(const StTensor& t) const { return files[t.file].base + files[t.file].data_off + t.begin; }
};

// Maps and indexes the files; a name present in two files is an error.
// Returns false with a message in `err`.
bool st_open(const std::vector<std::string>& paths, StCheckpoint& ck, std::string& err);

// The engine's name for a checkpoint name: prefixes some MLX exports carry
// ("language_model.", "model.language_model.") are removed so that decoder
// tensors read "model.layers.N...", "model.embed_tokens...", "model.norm...",
// "lm_head...".  Names outside the decoder map to an empty string.
std::string st_engine_name(const std::string& name);

// Parses one safetensors header (exposed for tests of malformed input).
bool st_parse_header(const char* json, size_t len, int file, std::vector<StTensor>& out, std::string& err);

}  // namespace iam

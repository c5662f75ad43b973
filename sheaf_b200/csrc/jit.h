// Compilation of generated kernel text to sm_100a cubins with NVRTC, with an
// on-disk cache keyed by the source text, compiler version and options.
#pragma once
#include <cstdint>
#include <map>
#include <string>
#include <vector>

namespace sb {

struct CubinChunk {
  std::string source;
  std::vector<uint8_t> cubin;
};

// Compiles each chunk (in parallel threads); throws std::runtime_error with the
// compiler log on failure.  Cache hits skip compilation.  With `prebuilt`
// (cubins by chunk key, from an ahead-of-time bundle) nothing is compiled: a
// chunk whose key is missing is an error.
using Prebuilt = std::map<std::string, std::vector<uint8_t>>;
void compile_chunks(std::vector<CubinChunk>& chunks, const std::string& cache_dir,
                    const Prebuilt* prebuilt = nullptr);

// Cache / bundle key of a chunk's source (compiler version and options included).
std::string chunk_key(const std::string& source);

// Default cache directory: $SHEAF_B200_CACHE, else <library dir>/kernel_cache.
std::string default_cache_dir();

// Splits a generated source made of independent kernel snippets into at most
// `max_chunks` compilation units of roughly equal size.
std::vector<CubinChunk> split_source(const std::vector<std::string>& snippets, const std::string& prelude,
                                     size_t max_chunks);

}  // namespace sb

// NVRTC compilation of generated kernels to sm_100a cubins, with a disk cache.
#include "jit.h"

#include <dlfcn.h>
#include <nvrtc.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <fstream>
#include <sstream>
#include <stdexcept>
#include <mutex>
#include <thread>

namespace sb {

namespace {

uint64_t fnv1a(const std::string& s, uint64_t h) {
  for (unsigned char c : s) {
    h ^= c;
    h *= 1099511628211ull;
  }
  return h;
}

const char* kOptions[] = {"--gpu-architecture=sm_100a", "--std=c++17", "-default-device",
                          "--fmad=true"};

std::string cache_key(const std::string& src) {
  int major = 0, minor = 0;
  nvrtcVersion(&major, &minor);
  std::string meta = "nvrtc" + std::to_string(major) + "." + std::to_string(minor);
  for (auto o : kOptions) meta += std::string(" ") + o;
  uint64_t a = fnv1a(meta + src, 1469598103934665603ull);
  uint64_t b = fnv1a(src + meta, 0x9e3779b97f4a7c15ull);
  char buf[40];
  std::snprintf(buf, sizeof buf, "%016llx%016llx", (unsigned long long)a, (unsigned long long)b);
  return buf;
}

bool read_file(const std::string& path, std::vector<uint8_t>* out) {
  std::ifstream f(path, std::ios::binary);
  if (!f) return false;
  out->assign(std::istreambuf_iterator<char>(f), std::istreambuf_iterator<char>());
  return !out->empty();
}

void write_file_atomic(const std::string& path, const std::vector<uint8_t>& data) {
  std::string tmp = path + ".tmp" + std::to_string(getpid()) + "_" +
                    std::to_string(std::hash<std::thread::id>()(std::this_thread::get_id()));
  {
    std::ofstream f(tmp, std::ios::binary);
    if (!f) return;
    f.write((const char*)data.data(), (std::streamsize)data.size());
  }
  std::rename(tmp.c_str(), path.c_str());
}

void mkdirs(const std::string& dir) {
  std::string cur;
  for (size_t i = 0; i < dir.size(); ++i) {
    cur += dir[i];
    if (dir[i] == '/' || i + 1 == dir.size()) mkdir(cur.c_str(), 0755);
  }
}

void compile_one(CubinChunk& ch, const std::string& cache_dir, std::string* err) {
  std::string key = cache_key(ch.source);
  std::string path = cache_dir.empty() ? "" : cache_dir + "/" + key + ".cubin";
  if (!path.empty() && read_file(path, &ch.cubin)) return;
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, ch.source.c_str(), "sheaf_b200_fused.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS) {
    *err = "nvrtcCreateProgram failed";
    return;
  }
  nvrtcResult r = nvrtcCompileProgram(prog, (int)(sizeof kOptions / sizeof *kOptions), kOptions);
  if (r != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    if (n) nvrtcGetProgramLog(prog, &log[0]);
    *err = std::string("NVRTC: ") + nvrtcGetErrorString(r) + "\n" + log.substr(0, 4000);
    nvrtcDestroyProgram(&prog);
    return;
  }
  size_t n = 0;
  nvrtcGetCUBINSize(prog, &n);
  ch.cubin.resize(n);
  nvrtcGetCUBIN(prog, (char*)ch.cubin.data());
  nvrtcDestroyProgram(&prog);
  if (!path.empty()) {
    mkdirs(cache_dir);
    write_file_atomic(path, ch.cubin);
  }
}

}  // namespace

std::string chunk_key(const std::string& source) { return cache_key(source); }

std::string default_cache_dir() {
  if (const char* e = std::getenv("SHEAF_B200_CACHE")) return e;
  Dl_info info;
  if (dladdr((void*)&default_cache_dir, &info) && info.dli_fname) {
    std::string p = info.dli_fname;
    auto k = p.rfind('/');
    if (k != std::string::npos) return p.substr(0, k) + "/kernel_cache";
  }
  return ".sheaf_b200_cache";
}

std::vector<CubinChunk> split_source(const std::vector<std::string>& snippets, const std::string& prelude,
                                     size_t max_chunks) {
  size_t total = 0;
  for (auto& s : snippets) total += s.size();
  size_t n = std::max<size_t>(1, std::min(max_chunks, snippets.size()));
  size_t target = total / n + 1;
  std::vector<CubinChunk> out;
  CubinChunk cur;
  cur.source = prelude;
  for (auto& s : snippets) {
    cur.source += s;
    if (cur.source.size() >= target && out.size() + 1 < n) {
      out.push_back(std::move(cur));
      cur = CubinChunk();
      cur.source = prelude;
    }
  }
  if (cur.source.size() > prelude.size() || out.empty()) out.push_back(std::move(cur));
  return out;
}

void compile_chunks(std::vector<CubinChunk>& chunks, const std::string& cache_dir, const Prebuilt* prebuilt) {
  if (prebuilt) {
    for (auto& ch : chunks) {
      auto it = prebuilt->find(cache_key(ch.source));
      if (it == prebuilt->end())
        throw std::runtime_error("the bundle has no cubin for a generated kernel chunk (built by another "
                                 "library version or for other options)");
      ch.cubin = it->second;
    }
    return;
  }
  std::vector<std::string> errs(chunks.size());
  unsigned hw = std::max(1u, std::thread::hardware_concurrency());
  size_t next = 0;
  std::vector<std::thread> ts;
  std::mutex mu;
  for (unsigned t = 0; t < std::min<size_t>(hw, chunks.size()); ++t) {
    ts.emplace_back([&]() {
      for (;;) {
        size_t i;
        {
          std::lock_guard<std::mutex> g(mu);
          if (next >= chunks.size()) return;
          i = next++;
        }
        compile_one(chunks[i], cache_dir, &errs[i]);
      }
    });
  }
  for (auto& t : ts) t.join();
  for (auto& e : errs)
    if (!e.empty()) throw std::runtime_error(e);
}

}  // namespace sb

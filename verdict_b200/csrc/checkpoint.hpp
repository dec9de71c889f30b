// Read-only safetensors checkpoints: one `model.safetensors`, or the shards
// listed by `model.safetensors.index.json`, memory-mapped; tensors are looked
// up by their state-dict names (HF Qwen3 / Qwen2 / Gemma decoders, the
// marker-head DecisionModel).  Format: 8-byte little-endian header length N,
// N bytes of JSON {name: {dtype, shape, data_offsets: [begin, end]}}, then the
// data; offsets are relative to the end of the header.
#pragma once

#include <dirent.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "json.hpp"

namespace vd {

enum StDtype : int { kStBF16 = 0, kStF16 = 1, kStF32 = 2 };

struct StTensor {
  int dtype = kStBF16;
  std::vector<int64_t> shape;
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t numel() const {
    int64_t n = 1;
    for (int64_t s : shape) n *= s;
    return n;
  }
};

class Checkpoint {
 public:
  explicit Checkpoint(const std::string& dir) {
    std::set<std::string> files;
    const std::string index = dir + "/model.safetensors.index.json";
    struct stat st;
    if (::stat(index.c_str(), &st) == 0) {
      const Json j = parse_json(read_text(index));
      if (!j.has("weight_map")) throw std::runtime_error("index without weight_map: " + index);
      for (const auto& kv : j.at("weight_map").obj) files.insert(kv.second.str);
    } else {
      DIR* d = ::opendir(dir.c_str());
      if (!d) throw std::runtime_error("cannot open checkpoint directory " + dir);
      while (dirent* e = ::readdir(d)) {
        const std::string n = e->d_name;
        if (n.size() > 12 && n.compare(n.size() - 12, 12, ".safetensors") == 0) files.insert(n);
      }
      ::closedir(d);
    }
    if (files.empty()) throw std::runtime_error("no .safetensors files in " + dir);
    for (const std::string& f : files) map_file(dir + "/" + f);
  }
  ~Checkpoint() {
    for (auto& m : maps_) ::munmap(m.first, m.second);
  }
  Checkpoint(const Checkpoint&) = delete;
  Checkpoint& operator=(const Checkpoint&) = delete;

  bool has(const std::string& name) const { return tensors_.count(name) != 0; }
  const StTensor& get(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) throw std::runtime_error("checkpoint has no tensor \"" + name + "\"");
    return it->second;
  }

 private:
  std::vector<std::pair<void*, size_t>> maps_;
  std::map<std::string, StTensor> tensors_;

  static std::string read_text(const std::string& path) {
    FILE* f = std::fopen(path.c_str(), "rb");
    if (!f) throw std::runtime_error("cannot read " + path);
    std::string s;
    char buf[65536];
    size_t n;
    while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) s.append(buf, n);
    std::fclose(f);
    return s;
  }

  void map_file(const std::string& path) {
    const int fd = ::open(path.c_str(), O_RDONLY);
    if (fd < 0) throw std::runtime_error("cannot open " + path);
    struct stat st;
    if (::fstat(fd, &st) != 0 || st.st_size < 8) {
      ::close(fd);
      throw std::runtime_error("bad safetensors file " + path);
    }
    const size_t size = static_cast<size_t>(st.st_size);
    void* base = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    ::close(fd);
    if (base == MAP_FAILED) throw std::runtime_error("mmap failed for " + path);
    maps_.emplace_back(base, size);
    const uint8_t* p = static_cast<const uint8_t*>(base);
    uint64_t hlen = 0;
    std::memcpy(&hlen, p, 8);  // little-endian hosts only
    if (hlen > size - 8) throw std::runtime_error("bad safetensors header in " + path);
    const Json h = parse_json(std::string(reinterpret_cast<const char*>(p + 8), hlen));
    const uint8_t* data = p + 8 + hlen;
    const size_t data_size = size - 8 - hlen;
    for (const auto& kv : h.obj) {
      if (kv.first == "__metadata__") continue;
      const Json& t = kv.second;
      StTensor x;
      const std::string dt = t.at("dtype").str;
      if (dt == "BF16") x.dtype = kStBF16;
      else if (dt == "F16") x.dtype = kStF16;
      else if (dt == "F32") x.dtype = kStF32;
      else throw std::runtime_error("tensor " + kv.first + " has unsupported dtype " + dt);
      for (const Json& d : t.at("shape").arr) x.shape.push_back(static_cast<int64_t>(d.num));
      const Json& off = t.at("data_offsets");
      const size_t b = static_cast<size_t>(off.arr.at(0).num), e = static_cast<size_t>(off.arr.at(1).num);
      const size_t esize = x.dtype == kStF32 ? 4 : 2;
      if (e < b || e > data_size || (e - b) != static_cast<size_t>(x.numel()) * esize)
        throw std::runtime_error("tensor " + kv.first + " has inconsistent offsets in " + path);
      x.data = data + b;
      x.nbytes = e - b;
      tensors_[kv.first] = x;
    }
  }
};

}  // namespace vd

// Reader for the *.safetensors shards of an mlx-lm converted checkpoint
// (the artifact format the reference loads in weights_loader.cc:72-154).
#pragma once

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace hyb {

struct TensorView {
    std::string dtype;              // "BF16", "U32", ...
    std::vector<int64_t> shape;
    const uint8_t* data = nullptr;  // points into a mapped shard
    size_t nbytes = 0;
};

// All tensors of every *.safetensors file in a directory (files mapped read-only
// for the lifetime of the object). Throws std::runtime_error / filesystem_error.
class Checkpoint {
  public:
    explicit Checkpoint(const std::string& dir);
    ~Checkpoint();
    Checkpoint(const Checkpoint&) = delete;
    Checkpoint& operator=(const Checkpoint&) = delete;

    bool has(const std::string& name) const { return tensors_.count(name) != 0; }
    const TensorView& get(const std::string& name) const;

  private:
    struct Mapping {
        void* addr = nullptr;
        size_t len = 0;
    };
    std::vector<Mapping> maps_;
    std::map<std::string, TensorView> tensors_;
};

}  // namespace hyb

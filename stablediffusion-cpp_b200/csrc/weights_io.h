// weights_io.h - host-side reading of .safetensors checkpoints (weights_io.cpp).
#pragma once

#include <cstdint>
#include <functional>
#include <string>
#include <vector>

namespace sdb {

// One tensor as read from a checkpoint: BF16 bit patterns or F32 values, row-major.
struct HostTensor {
  std::string name;
  bool bf16 = false;
  std::vector<int64_t> shape;
  std::vector<uint8_t> data;
};

// Tensor-parallel shard of this process: rank of world, with the model's head count.
struct TpShard {
  int rank = 0, world = 1, heads = 1;
};

// The files of <dir>/<base> as the reference's Weights::load_model finds them.
std::vector<std::string> checkpoint_files(const std::string& dir, const std::string& base);

// Calls sink once per F32 / F16 / BF16 tensor of `files`, converted as the reference
// converts (BF16 when keep_bf16 and numel >= min_numel, otherwise F32) and, when tp has
// world > 1, cut to tp->rank's Megatron shard (tensors other ranks own are skipped).
// With `only`, just the tensor of that name is converted (the others are skipped).
void read_checkpoint(const std::vector<std::string>& files, bool keep_bf16, int64_t min_numel, const TpShard* tp,
                     const std::function<void(HostTensor&&)>& sink, const std::string* only = nullptr);

// One named tensor of one file (no sharding); false if its dtype is not read.
bool read_tensor(const std::string& path, const std::string& name, bool keep_bf16, int64_t min_numel,
                 HostTensor& out);

}  // namespace sdb

// Host-side runtime pieces shared by the ensemble engine and single-layer handles:
// weight lookup by the reference's state_dict key names, a packed device weight
// arena, the slot-indexed recurrent-state table, and a scratch carver.
#pragma once
#include <functional>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "common.cuh"

namespace b2e {

// ------------------------------------------------------------- weights

struct HostTensor {
  const float* data = nullptr;
  int64_t numel = 0;
};

// Named host tensors as handed over the C-ABI. Lookups are strict, like
// load_state_dict(strict=True): a missing name or a wrong element count is an
// error, and so is a name that no module consumed (check_all_used).
class WeightSource {
 public:
  void add(const std::string& name, const float* data, int64_t numel);
  const float* get(const std::string& name, int64_t numel);
  void check_all_used() const;

 private:
  std::unordered_map<std::string, HostTensor> map_;
  std::unordered_set<std::string> used_;
};

// One device allocation holding every packed weight. Entries are planned with a
// fill callback, then filled into a single host buffer and uploaded in one copy.
// Entries of at most kSmallEntry bytes (norm weights, biases, conv taps, the 4x4
// BlockLinears) are packed together at the start of the allocation, the matrices
// after them from the next 2 MiB boundary. A step streams every matrix once,
// which evicts the GPU's address translations of the pages it passes; the small
// entries, which every per-row kernel reads, then share a few pages of their
// own instead of one page next to each matrix.
class WeightPack {
 public:
  static constexpr size_t kSmallEntry = 256 * 1024;
  ~WeightPack();
  // Returns the entry's offset, resolved by ptr() once upload() has run.
  size_t reserve(size_t bytes, std::function<void(uint8_t*)> fill);
  // Convenience packers (src is f32; `t` is the stored type).
  size_t add(const float* src, size_t n, int t);
  size_t add_rows(const std::vector<std::pair<const float*, size_t>>& parts, int t);  // concatenation
  size_t add_conv(const float* src, int channels, int taps);  // (C,1,taps) -> (taps, C)
  void upload();
  template <class T = void>
  T* ptr(size_t off) const {
    return reinterpret_cast<T*>(dev_ + ((off & kSmallTag) ? (off & ~kSmallTag) : big_base_ + off));
  }
  size_t bytes() const { return big_base_ + total_; }

 private:
  static constexpr size_t kSmallTag = size_t(1) << 62;  // offset bit: the entry is in the small region
  struct Entry {
    size_t off, bytes;
    std::function<void(uint8_t*)> fill;
  };
  std::vector<Entry> entries_;
  size_t total_ = 0;        // bytes of the matrix region
  size_t small_total_ = 0;  // bytes of the small region
  size_t big_base_ = 0;     // where the matrix region starts (set by upload)
  uint8_t* dev_ = nullptr;
};

void convert_f32(const float* src, void* dst, size_t n, int t);  // host f32 -> t (round to nearest even)

// ---------------------------------------------------------------- state

enum LeafKind : int { kLeafPlain = 0, kLeafConv = 1 };
enum LeafType : int { kLeafF32 = 0, kLeafI32 = 1 };

// One state leaf of one block: `elems` logical values per slot, stored in a
// leaf-major region with a 16-byte padded row stride. A conv window is stored
// tap-major (taps, C) so a row's channels are read coalesced; its exported
// layout is the reference's (C, taps) (model/modules.py:30-35).
struct Leaf {
  int kind = kLeafPlain, type = kLeafF32;
  int elems = 0, conv_c = 0, conv_taps = 0;
  long long stride = 0;  // 4-byte words per slot
  float init = 0.0f;
  size_t off = 0;        // byte offset of the region in the arena
};

class StateArena {
 public:
  ~StateArena();
  int add(int elems, int type = kLeafF32, float init = 0.0f);
  int add_conv(int channels, int taps);
  void allocate(int capacity);
  float* f32(int leaf) const { return reinterpret_cast<float*>(base_ + leaves_[leaf].off); }
  int* i32(int leaf) const { return reinterpret_cast<int*>(base_ + leaves_[leaf].off); }
  long long stride(int leaf) const { return leaves_[leaf].stride; }
  int capacity() const { return capacity_; }
  size_t bytes() const { return bytes_; }
  size_t slot_bytes() const;  // exported bytes of one slot (all leaves, reference layout)
  const std::vector<Leaf>& leaves() const { return leaves_; }
  void reset_all(cudaStream_t s);
  void reset_slots(const int* d_slots, int n, cudaStream_t s);  // device slot list
  void read_slot(int slot, void* host) const;                 // synchronous
  void write_slot(int slot, const void* host);                // synchronous

 private:
  std::vector<Leaf> leaves_;
  uint8_t* base_ = nullptr;
  size_t bytes_ = 0;
  int capacity_ = 0;
  struct DevLeaf { size_t off; long long stride; int elems; float init; };
  DevLeaf* dev_leaves_ = nullptr;
};

// --------------------------------------------------------------- scratch

// Carves one scratch allocation into 256-byte aligned buffers in a fixed order.
struct Carver {
  uint8_t* base = nullptr;  // null: size only
  size_t off = 0;
  template <class T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

}  // namespace b2e

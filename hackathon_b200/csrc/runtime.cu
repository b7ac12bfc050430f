#include <cmath>
#include <cstring>
#include <limits>

#include "runtime.cuh"

namespace b2e {

// ------------------------------------------------------------- weights

void WeightSource::add(const std::string& name, const float* data, int64_t numel) {
  B2E_CHECK(data != nullptr || numel == 0, kErrInvalid, "weight '" + name + "' has no data");
  B2E_CHECK(map_.emplace(name, HostTensor{data, numel}).second, kErrWeights, "duplicate weight '" + name + "'");
}

const float* WeightSource::get(const std::string& name, int64_t numel) {
  auto it = map_.find(name);
  B2E_CHECK(it != map_.end(), kErrWeights, "missing weight '" + name + "'");
  B2E_CHECK(it->second.numel == numel, kErrWeights,
            "weight '" + name + "' has " + std::to_string(it->second.numel) + " elements, expected " +
                std::to_string(numel));
  used_.insert(name);
  return it->second.data;
}

void WeightSource::check_all_used() const {
  for (const auto& kv : map_)
    B2E_CHECK(used_.count(kv.first), kErrWeights, "unexpected weight '" + kv.first + "'");
}

static uint16_t f32_to_bf16(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return uint16_t((u >> 16) | 0x40);  // NaN stays NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}

static uint16_t f32_to_f16(float f) {
  // Host round-to-nearest-even via the CUDA host-callable conversion.
  __half h = __float2half_rn(f);
  uint16_t r;
  std::memcpy(&r, &h, 2);
  return r;
}

void convert_f32(const float* src, void* dst, size_t n, int t) {
  if (t == kF32) {
    std::memcpy(dst, src, n * 4);
  } else if (t == kBF16) {
    auto* d = reinterpret_cast<uint16_t*>(dst);
    for (size_t i = 0; i < n; ++i) d[i] = f32_to_bf16(src[i]);
  } else {
    auto* d = reinterpret_cast<uint16_t*>(dst);
    for (size_t i = 0; i < n; ++i) d[i] = f32_to_f16(src[i]);
  }
}

WeightPack::~WeightPack() {
  if (dev_) cudaFree(dev_);
}

size_t WeightPack::reserve(size_t bytes, std::function<void(uint8_t*)> fill) {
  B2E_CHECK(dev_ == nullptr, kErrInternal, "weights reserved after upload");
  const bool small = bytes <= kSmallEntry;
  size_t& region = small ? small_total_ : total_;
  region = (region + 255) & ~size_t(255);
  const size_t off = region | (small ? kSmallTag : 0);
  entries_.push_back({off, bytes, std::move(fill)});
  region += bytes;
  return off;
}

size_t WeightPack::add(const float* src, size_t n, int t) {
  return reserve(n * dtype_size(t), [=](uint8_t* d) { convert_f32(src, d, n, t); });
}

size_t WeightPack::add_rows(const std::vector<std::pair<const float*, size_t>>& parts, int t) {
  size_t n = 0;
  for (auto& p : parts) n += p.second;
  return reserve(n * dtype_size(t), [=](uint8_t* d) {
    size_t o = 0;
    for (auto& p : parts) {
      convert_f32(p.first, d + o * dtype_size(t), p.second, t);
      o += p.second;
    }
  });
}

size_t WeightPack::add_conv(const float* src, int channels, int taps) {
  return reserve(size_t(channels) * taps * 4, [=](uint8_t* d) {
    float* o = reinterpret_cast<float*>(d);
    for (int c = 0; c < channels; ++c)
      for (int j = 0; j < taps; ++j) o[size_t(j) * channels + c] = src[size_t(c) * taps + j];
  });
}

void WeightPack::upload() {
  B2E_CHECK(dev_ == nullptr, kErrInternal, "weights uploaded twice");
  constexpr size_t kPage = size_t(2) << 20;
  big_base_ = (small_total_ + kPage - 1) / kPage * kPage;
  const size_t total = std::max<size_t>(big_base_ + total_, 256);
  std::vector<uint8_t> host(total, 0);
  for (auto& e : entries_)
    e.fill(host.data() + ((e.off & kSmallTag) ? (e.off & ~kSmallTag) : big_base_ + e.off));
  B2E_CUDA(cudaMalloc(&dev_, total));
  B2E_CUDA(cudaMemcpy(dev_, host.data(), total, cudaMemcpyHostToDevice));
  entries_.clear();
  entries_.shrink_to_fit();
}

// ---------------------------------------------------------------- state

StateArena::~StateArena() {
  if (base_) cudaFree(base_);
  if (dev_leaves_) cudaFree(dev_leaves_);
}

int StateArena::add(int elems, int type, float init) {
  Leaf l;
  l.kind = kLeafPlain;
  l.type = type;
  l.elems = elems;
  l.stride = (elems + 3) & ~3;
  l.init = init;
  leaves_.push_back(l);
  return int(leaves_.size()) - 1;
}

int StateArena::add_conv(int channels, int taps) {
  Leaf l;
  l.kind = kLeafConv;
  l.elems = channels * taps;
  l.conv_c = channels;
  l.conv_taps = taps;
  l.stride = (l.elems + 3) & ~3;
  leaves_.push_back(l);
  return int(leaves_.size()) - 1;
}

void StateArena::allocate(int capacity) {
  B2E_CHECK(capacity > 0, kErrInvalid, "state capacity must be positive");
  B2E_CHECK(base_ == nullptr, kErrInternal, "state allocated twice");
  capacity_ = capacity;
  size_t off = 0;
  for (auto& l : leaves_) {
    off = (off + 255) & ~size_t(255);
    l.off = off;
    off += size_t(capacity) * size_t(l.stride) * 4;
  }
  bytes_ = std::max<size_t>(off, 256);
  B2E_CUDA(cudaMalloc(&base_, bytes_));
  std::vector<DevLeaf> dl;
  for (auto& l : leaves_) dl.push_back({l.off, l.stride, l.elems, l.init});
  B2E_CUDA(cudaMalloc(&dev_leaves_, sizeof(DevLeaf) * std::max<size_t>(dl.size(), 1)));
  if (!dl.empty())
    B2E_CUDA(cudaMemcpy(dev_leaves_, dl.data(), sizeof(DevLeaf) * dl.size(), cudaMemcpyHostToDevice));
}

size_t StateArena::slot_bytes() const {
  size_t b = 0;
  for (auto& l : leaves_) b += size_t(l.elems) * 4;
  return b;
}

namespace {

struct DevLeafK { size_t off; long long stride; int elems; float init; };

// grid (slot-chunk, leaf); each thread fills words of one slot row.
__global__ void reset_rows_kernel(uint8_t* base, const DevLeafK* leaves, const int* slots, int n, int capacity) {
  const DevLeafK l = leaves[blockIdx.y];
  const uint32_t bits = __float_as_uint(l.init);
  const long long rows = slots ? n : capacity;
  const long long total = rows * l.stride;
  uint32_t* region = reinterpret_cast<uint32_t*>(base + l.off);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / l.stride, w = i - r * l.stride;
    const long long slot = slots ? slots[r] : r;
    if (slot < 0 || slot >= capacity) continue;
    region[slot * l.stride + w] = w < l.elems ? bits : 0u;
  }
}

}  // namespace

void StateArena::reset_all(cudaStream_t s) {
  if (leaves_.empty()) return;
  dim3 grid(1024, unsigned(leaves_.size()));
  reset_rows_kernel<<<grid, 256, 0, s>>>(base_, reinterpret_cast<const DevLeafK*>(dev_leaves_), nullptr, 0,
                                         capacity_);
  B2E_CUDA(cudaGetLastError());
}

void StateArena::reset_slots(const int* d_slots, int n, cudaStream_t s) {
  if (leaves_.empty() || n <= 0) return;
  dim3 grid(std::min(1024, ceil_div(long(n) * 64, 256)), unsigned(leaves_.size()));
  reset_rows_kernel<<<grid, 256, 0, s>>>(base_, reinterpret_cast<const DevLeafK*>(dev_leaves_), d_slots, n,
                                         capacity_);
  B2E_CUDA(cudaGetLastError());
}

void StateArena::read_slot(int slot, void* host) const {
  B2E_CHECK(slot >= 0 && slot < capacity_, kErrCapacity, "slot out of range");
  uint8_t* out = reinterpret_cast<uint8_t*>(host);
  std::vector<float> tmp;
  for (auto& l : leaves_) {
    const size_t nb = size_t(l.elems) * 4;
    const uint8_t* src = base_ + l.off + size_t(slot) * l.stride * 4;
    if (l.kind == kLeafConv) {
      tmp.resize(l.elems);
      B2E_CUDA(cudaMemcpy(tmp.data(), src, nb, cudaMemcpyDeviceToHost));
      float* o = reinterpret_cast<float*>(out);
      for (int c = 0; c < l.conv_c; ++c)
        for (int j = 0; j < l.conv_taps; ++j) o[c * l.conv_taps + j] = tmp[size_t(j) * l.conv_c + c];
    } else {
      B2E_CUDA(cudaMemcpy(out, src, nb, cudaMemcpyDeviceToHost));
    }
    out += nb;
  }
}

void StateArena::write_slot(int slot, const void* host) {
  B2E_CHECK(slot >= 0 && slot < capacity_, kErrCapacity, "slot out of range");
  const uint8_t* in = reinterpret_cast<const uint8_t*>(host);
  std::vector<float> tmp;
  for (auto& l : leaves_) {
    const size_t nb = size_t(l.elems) * 4;
    uint8_t* dst = base_ + l.off + size_t(slot) * l.stride * 4;
    if (l.kind == kLeafConv) {
      tmp.resize(l.elems);
      const float* s = reinterpret_cast<const float*>(in);
      for (int c = 0; c < l.conv_c; ++c)
        for (int j = 0; j < l.conv_taps; ++j) tmp[size_t(j) * l.conv_c + c] = s[c * l.conv_taps + j];
      B2E_CUDA(cudaMemcpy(dst, tmp.data(), nb, cudaMemcpyHostToDevice));
    } else {
      B2E_CUDA(cudaMemcpy(dst, in, nb, cudaMemcpyHostToDevice));
    }
    in += nb;
  }
}

}  // namespace b2e

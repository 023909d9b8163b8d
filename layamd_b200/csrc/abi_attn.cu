// Kernel-level C entry point for the encoder attention on caller-owned device buffers: the attention
// parity tests and the isolated attention benchmark use it. An addition to the reference ABI; the
// engine itself never calls it.
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <vector>

#include "kernels.h"
#include "laya_api.h"

namespace {
std::mutex g_mu;
struct AttnDev {
  bool ready = false;
  int* ticket = nullptr;   // work / exit counters of the persistent tcgen05 kernel (kept zero between launches)
  int* meta = nullptr;     // soff[B] | slen[B] | items (4 ints each)
  size_t meta_ints = 0;
};
std::vector<AttnDev> g_dev;
}  // namespace

extern "C" int laya_b200_attention(const void* qkv, void* out, int rows, int B, const int* lens, int H, int window,
                                   int impl, void* stream, int sync) {
  using namespace laya;
  if (!qkv || !out || !lens || B <= 0 || H <= 0 || rows <= 0 || window < 0 || (impl != 0 && impl != 1)) return -2;
  long long total = 0;
  for (int i = 0; i < B; ++i) {
    if (lens[i] <= 0) return -2;
    total += lens[i];
  }
  if (total > rows) return -2;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  const int qrows = impl == 0 ? 128 : 64;
  std::vector<int> meta((2 * (size_t)B + 3) & ~size_t(3));  // items start 16-byte aligned
  std::vector<AttnItem> items;
  int off = 0;
  for (int i = 0; i < B; ++i) {
    meta[i] = off;
    meta[B + i] = lens[i];
    for (int q0 = 0; q0 < lens[i]; q0 += qrows) items.push_back(AttnItem{i, q0, off, lens[i]});
    off += lens[i];
  }
  if (impl == 0)  // the tcgen05 kernel hands units out longest sequence first, as the engine orders them
    std::stable_sort(items.begin(), items.end(), [](const AttnItem& x, const AttnItem& y) { return x.nq > y.nq; });
  const size_t n_ints = meta.size() + items.size() * 4;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int* d_meta;
  int* err;
  int* ticket;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if ((int)g_dev.size() <= dev) g_dev.resize(dev + 1);
    AttnDev& d = g_dev[dev];
    if (!d.ready) {
      if (attn_tc_prepare_device() != cudaSuccess) return -4;
      if (cudaMalloc(&d.ticket, 2 * sizeof(int)) != cudaSuccess) return -4;
      if (cudaMemset(d.ticket, 0, 2 * sizeof(int)) != cudaSuccess) return -4;
      d.ready = true;
    }
    if (d.meta_ints < n_ints) {
      if (d.meta) cudaFree(d.meta);
      d.meta = nullptr;
      d.meta_ints = 0;
      if (cudaMalloc(&d.meta, n_ints * sizeof(int)) != cudaSuccess) return -4;
      d.meta_ints = n_ints;
    }
    d_meta = d.meta;
    ticket = d.ticket;
  }
  err = entry_error_word(dev);
  if (!err) return -4;
  // the previous call may still read the metadata block: order the upload after it on the stream
  if (cudaMemcpyAsync(d_meta, meta.data(), meta.size() * sizeof(int), cudaMemcpyHostToDevice, st) != cudaSuccess ||
      cudaMemcpyAsync(d_meta + meta.size(), items.data(), items.size() * sizeof(AttnItem), cudaMemcpyHostToDevice,
                      st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return -5;
  AttnArgs a;
  a.qkv = qkv;
  a.out = out;
  a.out_plane = 0;
  a.out_planes = 1;
  a.items = reinterpret_cast<const AttnItem*>(d_meta + meta.size());
  a.n_items = static_cast<int>(items.size());
  a.soff = d_meta;
  a.slen = d_meta + B;
  a.gsrc = nullptr;
  a.gdst = nullptr;
  a.gathered = 0;
  a.H = H;
  a.window = window;
  a.scale = 0.125f;
  cudaError_t e;
  if (impl == 0) {
    CUtensorMap tq, tkv;
    if (!make_operand_map(&tq, qkv, 3ull * 64 * H, (uint64_t)rows, 1, 128) ||
        !make_operand_map(&tkv, qkv, 3ull * 64 * H, (uint64_t)rows, 1, 64))
      return -3;
    e = attn_tc_launch(tq, tkv, a, ticket, err, st);
  } else {
    e = attn_bf16_launch(a, st);
  }
  if (e != cudaSuccess) {
    fprintf(stderr, "[laya] attention launch: %s\n", cudaGetErrorString(e));
    return -5;
  }
  if (sync) {
    if (cudaStreamSynchronize(st) != cudaSuccess) return -6;
    int h = 0;
    cudaMemcpy(&h, err, sizeof(int), cudaMemcpyDeviceToHost);
    if (h) {
      cudaMemset(err, 0, sizeof(int));
      // an aborted launch can leave the work / exit counters part-way: clear them for the next call
      cudaMemset(ticket, 0, 2 * sizeof(int));
      return -100 - h;
    }
  }
  return 0;
}

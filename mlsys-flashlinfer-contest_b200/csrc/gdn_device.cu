// Per-device facts the launchers need: the SM count of the current device and
// the one-time opt-in to more than 48 KiB of dynamic shared memory per kernel.
// Both are per device (a process may drive several GPUs, one per host thread or
// by switching the current device), cached, and safe to call from any thread.
#include <atomic>
#include <mutex>

#include "gdn_internal.h"

namespace gdn {

namespace {
constexpr int kMaxDevices = 64;
constexpr int kDefaultSms = 148;  // B200; used only if the attribute query fails

std::atomic<int> g_sms[kMaxDevices];  // 0 = not queried yet

struct AttrEntry {
  int dev;
  const void* func;
  int bytes;
};
constexpr int kMaxAttrEntries = 256;
std::mutex g_attr_mu;
AttrEntry g_attr[kMaxAttrEntries];
int g_attr_used = 0;
}  // namespace

int device_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return kDefaultSms;
  if (dev >= kMaxDevices) {
    int v = 0;
    return cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0
               ? v
               : kDefaultSms;
  }
  int v = g_sms[dev].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
    v = kDefaultSms;
  g_sms[dev].store(v, std::memory_order_relaxed);
  return v;
}

cudaError_t set_max_dynamic_smem(const void* func, int bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_attr_mu);
  for (int i = 0; i < g_attr_used; ++i)
    if (g_attr[i].dev == dev && g_attr[i].func == func && g_attr[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  if (g_attr_used < kMaxAttrEntries) g_attr[g_attr_used++] = AttrEntry{dev, func, bytes};
  return cudaSuccess;
}

}  // namespace gdn

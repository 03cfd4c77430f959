// Per-device SM counts and per-(kernel, device) shared-memory attributes (device_info.h).
#include <map>
#include <mutex>
#include <utility>

#include "device_info.h"

namespace kimi {
namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mutex;
int g_sms[kMaxDevices] = {};
std::map<std::pair<const void*, int>, int>* g_smem = nullptr;  // (kernel, device) -> bytes set

}  // namespace

int device_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (g_sms[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sms[dev] = n;
  }
  return g_sms[dev];
}

cudaError_t ensure_dynamic_smem(const void* kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(g_mutex);
  if (!g_smem) g_smem = new std::map<std::pair<const void*, int>, int>();
  auto it = g_smem->find({kernel, dev});
  if (it != g_smem->end() && it->second >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  (*g_smem)[{kernel, dev}] = bytes;
  return cudaSuccess;
}

}  // namespace kimi

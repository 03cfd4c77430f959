// Per-device facts and one-time kernel set-up shared by the host-side launchers.
//
// A process may drive several GPUs (a serving process with one stream per device, a test that
// walks every visible device), so nothing here is cached per process: each value or setting is
// keyed by the device that is current on the calling host thread.
#pragma once
#include <cuda_runtime.h>

namespace kimi {

// Streaming multiprocessors of the current device (queried once per device).
int device_sms();

// Raise `kernel`'s dynamic shared-memory limit to at least `bytes` on the current device.  The
// attribute is set once per (kernel, device) pair; later calls are a locked table lookup.
cudaError_t ensure_dynamic_smem(const void* kernel, int bytes);

template <typename K>
inline cudaError_t ensure_dynamic_smem(K* kernel, int bytes) {
  return ensure_dynamic_smem(reinterpret_cast<const void*>(kernel), bytes);
}

}  // namespace kimi

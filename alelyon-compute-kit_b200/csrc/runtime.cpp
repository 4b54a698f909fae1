// The C ABI of libalelyon_compute_kit.so over the CUDA runtime.
//
// Restates the contract of the reference's Rust C ABI (ffi.rs) for the core
// device entries and the vq4 extension, B200-first:
//   * a device is one CUDA device with one non-blocking stream; operator
//     entries enqueue on it and return ACK_OK (= accepted, not finished);
//     ack_download waits for the stream, so a readback sees all earlier work
//     (ffi.rs:48-64);
//   * handles are ids looked up in a registry under a lock, never
//     dereferenced (ffi.rs:10-25); a buffer handle is (device id << 32) | seq;
//   * one mutex per device serialises calls on it (ffi.rs:27-34);
//   * a CUDA error that leaves the context unusable (an illegal address, a
//     launch failure) poisons the device: every later call on it refuses
//     with ACK_ERR_POISONED, a free leaks and counts its buffer, close still
//     succeeds (ffi.rs:16-20);
//   * the last error message is per thread (ffi.rs:1368).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>

#include "alelyon_compute_kit.h"
#include "vq_kernels.hpp"
#include "vq_plan.hpp"

#define ACK_EXPORT extern "C" __attribute__((visibility("default")))

namespace {

thread_local std::string g_last_error;

void set_error(const std::string& m) { g_last_error = m; }

std::string format(const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  return buf;
}

struct BufferRec {
  void* ptr = nullptr;
  uint64_t bytes = 0;
  uint64_t id = 0;
};

struct Device {
  uint64_t id = 0;
  int ordinal = 0;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  bool closed = false;
  bool poisoned = false;
  std::unordered_map<uint32_t, BufferRec> buffers;
  uint32_t next_buffer = 1;
  uint64_t leaked = 0;
  cudaDeviceProp prop{};
  int inject_sync = 0;       // test-only: error reported by the next synchronisation
  bool inject_alloc = false; // test-only: the next allocation reports failure
  // the copy streams, events and device scratch of ack_vq2_dense_host,
  // created on first use; the scratch grows to the largest call's need and
  // is kept until close (returning it to the driver on every call costs
  // milliseconds of page mapping per call)
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t ev[7] = {};    // allocated, h_done[2], k_done[2], d_done[2]
  void* scratch = nullptr;
  uint64_t scratch_bytes = 0;
};

struct Registry {
  std::mutex mu;
  std::unordered_map<uint64_t, std::shared_ptr<Device>> devices;
  uint64_t next_device = 1;
};

Registry& registry() {
  static Registry* r = new Registry;  // never destroyed: no teardown-order hazards at exit
  return *r;
}

// Make `ordinal` current for the scope and restore the caller's device after.
class DeviceScope {
 public:
  explicit DeviceScope(int ordinal) {
    if (cudaGetDevice(&prev_) != cudaSuccess) prev_ = -1;
    if (prev_ != ordinal) cudaSetDevice(ordinal);
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev_ >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = -1;
};

// Errors after which the CUDA context cannot be trusted.
bool sticky(cudaError_t e) {
  switch (e) {
    case cudaErrorIllegalAddress:
    case cudaErrorLaunchFailure:
    case cudaErrorHardwareStackError:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorInvalidAddressSpace:
    case cudaErrorInvalidPc:
    case cudaErrorAssert:
    case cudaErrorLaunchTimeout:
    case cudaErrorECCUncorrectable:
    case cudaErrorContextIsDestroyed:
    case cudaErrorDevicesUnavailable:
    case cudaErrorUnknown:
      return true;
    default:
      return false;
  }
}

int32_t cuda_fail(Device& d, cudaError_t e, const char* what) {
  set_error(format("%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e)));
  if (sticky(e)) {
    d.poisoned = true;
    return ACK_ERR_POISONED;
  }
  return ACK_ERR_VULKAN;
}

int32_t lookup(const AckDevice* handle, std::shared_ptr<Device>* out) {
  const uint64_t id = uint64_t(reinterpret_cast<uintptr_t>(handle));
  if (!id) {
    set_error("null device handle");
    return ACK_ERR_NULL;
  }
  Registry& r = registry();
  std::lock_guard<std::mutex> lk(r.mu);
  auto it = r.devices.find(id);
  if (it == r.devices.end()) {
    set_error(format("device handle %llu is not open (closed, never opened, or not a kit handle)",
                     (unsigned long long)id));
    return ACK_ERR_CLOSED;
  }
  *out = it->second;
  return ACK_OK;
}

// The device lock, or ACK_ERR_CLOSED once closed (ffi.rs:1906-1916).
int32_t acquire(Device& d, std::unique_lock<std::mutex>* lk) {
  *lk = std::unique_lock<std::mutex>(d.mu);
  if (d.closed) {
    set_error(format("device %llu is closed", (unsigned long long)d.id));
    return ACK_ERR_CLOSED;
  }
  return ACK_OK;
}

// A buffer handle resolved against the device that must own it (ffi.rs:1919-1941).
int32_t buffer_of(Device& d, const AckBuffer* handle, BufferRec** out) {
  const uint64_t raw = uint64_t(reinterpret_cast<uintptr_t>(handle));
  if (!raw) {
    set_error("null buffer handle");
    return ACK_ERR_NULL;
  }
  const uint64_t owner = raw >> 32;
  const uint32_t seq = uint32_t(raw & 0xffffffffu);
  if (owner != d.id) {
    set_error(format("buffer %#llx belongs to device %llu, not device %llu", (unsigned long long)raw,
                     (unsigned long long)owner, (unsigned long long)d.id));
    return ACK_ERR_FOREIGN;
  }
  auto it = d.buffers.find(seq);
  if (it == d.buffers.end()) {
    set_error(format("buffer %#llx is not live on device %llu (freed, or never allocated)", (unsigned long long)raw,
                     (unsigned long long)d.id));
    return ACK_ERR_FREED;
  }
  *out = &it->second;
  return ACK_OK;
}

int32_t refuse_poisoned(const Device& d, const char* what) {
  if (!d.poisoned) return ACK_OK;
  set_error(format("%s: device %llu poisoned by an earlier failed CUDA operation; close it", what,
                   (unsigned long long)d.id));
  return ACK_ERR_POISONED;
}

// Wait for the device stream; a test-only injected fault reports after the real wait.
cudaError_t sync_stream(Device& d) {
  cudaError_t e = cudaStreamSynchronize(d.stream);
  if (e == cudaSuccess && d.inject_sync) {
    e = cudaError_t(d.inject_sync);
    d.inject_sync = 0;
  }
  return e;
}

uint64_t fnv1a(const void* data, size_t len, uint64_t h = 0xcbf29ce484222325ull) {
  const unsigned char* p = static_cast<const unsigned char*>(data);
  for (size_t i = 0; i < len; ++i) {
    h ^= p[i];
    h *= 0x100000001b3ull;
  }
  return h;
}

#include "manifest.inc"

// FNV-1a over the embedded kernel manifest (sources' sha256, compiler, flags).
uint64_t shader_identity() { return fnv1a(kManifestJson, sizeof(kManifestJson) - 1); }

constexpr const char* kVersion = "alelyon-compute-kit-b200 0.1.0";
constexpr uint64_t kPoolKeepBytes = uint64_t(1) << 30;  // freed buffer memory the pool keeps cached

int32_t plan_refused(const char* entry, ack::PlanError e, int schema, int slot) {
  set_error(format("%s: plan refused: %s", entry, ack::plan_error_name(e, schema, slot).c_str()));
  return ack::plan_error_code(e);
}

// ACK_DEVICE: "gpu", "gpu:<n>", "any", "any:<n>" choose a CUDA ordinal
// (device_choice.rs:11-22); "cpu" is refused; unset = the current device.
int choose_ordinal(std::string* why) {
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count == 0) {
    *why = format("no CUDA device: %s", e == cudaSuccess ? "none found" : cudaGetErrorString(e));
    return -1;
  }
  const char* env = getenv("ACK_DEVICE");
  if (!env || !*env) {
    int cur = 0;
    if (cudaGetDevice(&cur) != cudaSuccess) cur = 0;
    return cur;
  }
  std::string s(env);
  std::string kind = s.substr(0, s.find(':'));
  if (kind == "cpu") {
    *why = "ACK_DEVICE=cpu: this build has no CPU device; the vq4 path runs on CUDA only";
    return -1;
  }
  if (kind != "gpu" && kind != "any") {
    *why = format("ACK_DEVICE=%s is not gpu, gpu:<n>, any or any:<n>", env);
    return -1;
  }
  int n = 0;
  if (s.find(':') != std::string::npos) {
    char* end = nullptr;
    long v = strtol(s.c_str() + s.find(':') + 1, &end, 10);
    if (!end || *end || v < 0) {
      *why = format("ACK_DEVICE=%s: the ordinal is not a number", env);
      return -1;
    }
    n = int(v);
  }
  if (n >= count) {
    *why = format("ACK_DEVICE=%s: only %d CUDA device(s)", env, count);
    return -1;
  }
  return n;
}

}  // namespace

// ------------------------------------------------------------- core entries --

ACK_EXPORT int32_t ack_abi_info(AckAbiInfo* out, size_t size) {
  if (!out) return ACK_ERR_NULL;
  if (size < sizeof(AckAbiInfo)) {
    set_error(format("AckAbiInfo of %zu bytes is smaller than this library's %zu", size, sizeof(AckAbiInfo)));
    return ACK_ERR_ABI;
  }
  AckAbiInfo info;
  memset(&info, 0, sizeof(info));
  info.size = sizeof(AckAbiInfo);
  info.version = ACK_ABI_VERSION;
  info.operators = 0;  // none of the reference's dense operator families
  info.shaders = shader_identity();
  uint64_t b = fnv1a(kVersion, strlen(kVersion));
  info.build = fnv1a(&info.shaders, sizeof(info.shaders), b);
  memcpy(out, &info, sizeof(info));
  return ACK_OK;
}

ACK_EXPORT AckDevice* ack_open(void) {
  std::string why;
  const int ordinal = choose_ordinal(&why);
  if (ordinal < 0) {
    set_error(why);
    return nullptr;
  }
  auto dev = std::make_shared<Device>();
  dev->ordinal = ordinal;
  {
    DeviceScope scope(ordinal);
    cudaError_t e = cudaGetDeviceProperties(&dev->prop, ordinal);
    if (e != cudaSuccess) {
      set_error(format("ack_open: %s", cudaGetErrorString(e)));
      return nullptr;
    }
    if (dev->prop.major != 10 || dev->prop.minor != 0) {
      set_error(format("ack_open: this library is built for sm_100a (B200); CUDA device %d is sm_%d%d", ordinal,
                       dev->prop.major, dev->prop.minor));
      return nullptr;
    }
    e = cudaStreamCreateWithFlags(&dev->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
      set_error(format("ack_open: stream: %s", cudaGetErrorString(e)));
      return nullptr;
    }
    // Buffers come from the device's stream-ordered pool (cudaMallocAsync on
    // the device stream): a free neither waits for the whole device nor, up
    // to this much cached memory, hands pages back to the driver.
    cudaMemPool_t pool = nullptr;
    if (cudaDeviceGetDefaultMemPool(&pool, ordinal) == cudaSuccess) {
      uint64_t threshold = 0;
      if (cudaMemPoolGetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold) == cudaSuccess &&
          threshold < kPoolKeepBytes) {
        threshold = kPoolKeepBytes;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold);
      }
    }
    cudaGetLastError();
  }
  Registry& r = registry();
  std::lock_guard<std::mutex> lk(r.mu);
  if (r.next_device > 0xffffffffull) {
    set_error("device handle space exhausted in this process");
    DeviceScope scope(ordinal);
    cudaStreamDestroy(dev->stream);
    return nullptr;
  }
  dev->id = r.next_device++;
  r.devices[dev->id] = dev;
  return reinterpret_cast<AckDevice*>(uintptr_t(dev->id));
}

ACK_EXPORT int32_t ack_close(AckDevice* handle) {
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  {
    std::unique_lock<std::mutex> lk;
    rc = acquire(*dev, &lk);
    if (rc) return rc;
    if (!dev->buffers.empty()) {
      set_error(format("close refused: %zu buffer(s) still allocated on this device", dev->buffers.size()));
      return ACK_ERR_LIVE_BUFFERS;
    }
    if (!dev->poisoned) {
      DeviceScope scope(dev->ordinal);
      cudaError_t e = sync_stream(*dev);
      if (e != cudaSuccess) {
        set_error(format("close waited for enqueued work and it failed: %s", cudaGetErrorString(e)));
      } else {
        cudaStreamDestroy(dev->stream);
        for (cudaStream_t st : {dev->copy_in, dev->copy_out})
          if (st) cudaStreamDestroy(st);
        for (cudaEvent_t ev : dev->ev)
          if (ev) cudaEventDestroy(ev);
        if (dev->scratch) cudaFree(dev->scratch);
        dev->scratch = nullptr;
        dev->scratch_bytes = 0;
      }
    }
    dev->closed = true;
  }
  Registry& r = registry();
  std::lock_guard<std::mutex> lk(r.mu);
  r.devices.erase(dev->id);
  return ACK_OK;
}

ACK_EXPORT int32_t ack_device_info(const AckDevice* handle, AckDeviceInfo* out, size_t size) {
  if (!out) return ACK_ERR_NULL;
  if (size < sizeof(AckDeviceInfo)) {
    set_error(format("AckDeviceInfo of %zu bytes is smaller than this library's %zu", size, sizeof(AckDeviceInfo)));
    return ACK_ERR_ABI;
  }
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  const cudaDeviceProp& p = dev->prop;
  AckDeviceInfo info;
  memset(&info, 0, sizeof(info));
  info.size = sizeof(AckDeviceInfo);
  info.version = ACK_DEVICE_INFO_VERSION;
  int runtime = 0, driver = 0;
  cudaRuntimeGetVersion(&runtime);
  cudaDriverGetVersion(&driver);
  // Vulkan-style packed version (major << 22 | minor << 12) of the CUDA runtime
  info.api_version = (uint32_t(runtime / 1000) << 22) | (uint32_t((runtime % 1000) / 10) << 12);
  info.driver_version_raw = uint32_t(driver);
  info.driver_id = 0;
  info.vendor_id = 0x10DE;
  info.device_id = uint32_t(p.pciDeviceID);
  info.device_type = 2;  // a discrete GPU
  memcpy(info.device_uuid, p.uuid.bytes, 16);
  info.features = 0;
  info.subgroup_size = uint32_t(p.warpSize);
  info.timestamp_valid_bits = 64;
  info.timestamp_period_ns = 1.0f;
  info.max_push_constant_bytes = 32764;  // kernel parameter space
  info.device_local_bytes = p.totalGlobalMem;
  info.max_storage_buffer_bytes = p.totalGlobalMem;
  info.max_workgroup_invocations = uint32_t(p.maxThreadsPerBlock);
  for (int i = 0; i < 3; ++i) {
    info.max_workgroup_count[i] = uint32_t(p.maxGridSize[i]);
    info.max_workgroup_size[i] = uint32_t(p.maxThreadsDim[i]);
  }
  uint64_t id = fnv1a(reinterpret_cast<const unsigned char*>(&info) + 8, 152);
  uint64_t sh = shader_identity();
  info.identity = fnv1a(&sh, sizeof(sh), id);
  snprintf(info.device_name, sizeof(info.device_name), "%s", p.name);
  snprintf(info.driver_name, sizeof(info.driver_name), "NVIDIA CUDA");
  snprintf(info.driver_info, sizeof(info.driver_info), "driver API %d.%d, runtime %d.%d, sm_%d%d, %d SMs",
           driver / 1000, (driver % 1000) / 10, runtime / 1000, (runtime % 1000) / 10, p.major, p.minor,
           p.multiProcessorCount);
  memcpy(out, &info, sizeof(info));
  return ACK_OK;
}

ACK_EXPORT int32_t ack_device_name(const AckDevice* handle, char* out, size_t len) {
  if (!out || len == 0) return ACK_ERR_NULL;
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  const size_t n = std::min(strlen(dev->prop.name), len - 1);
  memcpy(out, dev->prop.name, n);
  out[n] = 0;
  return ACK_OK;
}

ACK_EXPORT int32_t ack_live_objects(const AckDevice* handle, int64_t* out) {
  if (!out) return ACK_ERR_NULL;
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  *out = 1 + int64_t(dev->buffers.size()) + int64_t(dev->leaked);
  return ACK_OK;
}

ACK_EXPORT int32_t ack_leaked_on_poison(const AckDevice* handle, uint64_t* out) {
  if (!out) return ACK_ERR_NULL;
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  *out = dev->leaked;
  return ACK_OK;
}

ACK_EXPORT int32_t ack_last_error(char* out, size_t len) {
  if (!out || len == 0) return ACK_ERR_NULL;
  const size_t n = std::min(g_last_error.size(), len - 1);
  memcpy(out, g_last_error.data(), n);
  out[n] = 0;
  return ACK_OK;
}

ACK_EXPORT AckBuffer* ack_buffer_alloc(const AckDevice* handle, uint64_t bytes) {
  if (bytes == 0) {
    set_error("zero-byte buffer");
    return nullptr;
  }
  std::shared_ptr<Device> dev;
  if (lookup(handle, &dev)) return nullptr;
  std::unique_lock<std::mutex> lk;
  if (acquire(*dev, &lk)) return nullptr;
  if (refuse_poisoned(*dev, "buffer alloc")) return nullptr;
  if (dev->next_buffer == 0xffffffffu) {
    set_error("buffer handle space exhausted on this device; close and reopen");
    return nullptr;
  }
  DeviceScope scope(dev->ordinal);
  void* ptr = nullptr;
  // stream-ordered: usable by everything later enqueued on the device stream
  cudaError_t e = cudaMallocAsync(&ptr, bytes, dev->stream);
  if (e == cudaSuccess && dev->inject_alloc) {
    dev->inject_alloc = false;
    cudaFreeAsync(ptr, dev->stream);
    ptr = nullptr;
    e = cudaErrorMemoryAllocation;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();  // an allocation failure is not sticky; clear it
    set_error(format("buffer alloc of %llu bytes: %s (%s)", (unsigned long long)bytes, cudaGetErrorName(e),
                     cudaGetErrorString(e)));
    if (sticky(e)) dev->poisoned = true;
    return nullptr;
  }
  const uint32_t seq = dev->next_buffer++;
  const uint64_t h = (dev->id << 32) | seq;
  dev->buffers[seq] = BufferRec{ptr, bytes, h};
  return reinterpret_cast<AckBuffer*>(uintptr_t(h));
}

ACK_EXPORT int32_t ack_buffer_free(const AckDevice* handle, AckBuffer* buf) {
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  BufferRec* b = nullptr;
  rc = buffer_of(*dev, buf, &b);
  if (rc) return rc;
  const uint32_t seq = uint32_t(uint64_t(reinterpret_cast<uintptr_t>(buf)) & 0xffffffffu);
  void* ptr = b->ptr;
  dev->buffers.erase(seq);
  if (dev->poisoned) {
    // the handle is consumed; the allocation is left alone and counted
    dev->leaked += 1;
    set_error("buffer leaked, not freed: the device is poisoned");
    return ACK_ERR_POISONED;
  }
  DeviceScope scope(dev->ordinal);
  cudaError_t e = cudaFreeAsync(ptr, dev->stream);  // after the enqueued work that may still use it
  if (e != cudaSuccess) return cuda_fail(*dev, e, "buffer free");
  return ACK_OK;
}

ACK_EXPORT int32_t ack_upload(const AckDevice* handle, const AckBuffer* buf, const void* data, size_t len) {
  if (!data) return ACK_ERR_NULL;
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  BufferRec* b = nullptr;
  rc = buffer_of(*dev, buf, &b);
  if (rc) return rc;
  if (uint64_t(len) != b->bytes) {
    set_error(format("upload of %zu bytes into a %llu-byte buffer", len, (unsigned long long)b->bytes));
    return ACK_ERR_SIZE;
  }
  rc = refuse_poisoned(*dev, "upload");
  if (rc) return rc;
  DeviceScope scope(dev->ordinal);
  cudaError_t e = cudaMemcpyAsync(b->ptr, data, len, cudaMemcpyHostToDevice, dev->stream);
  if (e == cudaSuccess) e = sync_stream(*dev);  // the caller's bytes may go away on return
  if (e != cudaSuccess) return cuda_fail(*dev, e, "upload");
  return ACK_OK;
}

ACK_EXPORT int32_t ack_download(const AckDevice* handle, const AckBuffer* buf, void* data, size_t len) {
  if (!data) return ACK_ERR_NULL;
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  BufferRec* b = nullptr;
  rc = buffer_of(*dev, buf, &b);
  if (rc) return rc;
  if (uint64_t(len) != b->bytes) {
    set_error(format("download of %zu bytes from a %llu-byte buffer", len, (unsigned long long)b->bytes));
    return ACK_ERR_SIZE;
  }
  rc = refuse_poisoned(*dev, "download");
  if (rc) return rc;
  DeviceScope scope(dev->ordinal);
  cudaError_t e = cudaMemcpyAsync(data, b->ptr, len, cudaMemcpyDeviceToHost, dev->stream);
  if (e == cudaSuccess) e = sync_stream(*dev);
  if (e != cudaSuccess) return cuda_fail(*dev, e, "download");
  return ACK_OK;
}

ACK_EXPORT int32_t ack_inject_fault(const AckDevice* handle, int32_t kind, int32_t code) {
  const char* env = getenv("ACK_FAULT_INJECTION");
  if (!env || strcmp(env, "1") != 0) {
    set_error("ack_inject_fault: fault injection is disabled in this process (set ACK_FAULT_INJECTION=1)");
    return ACK_ERR_UNSUPPORTED_OP;
  }
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  if (kind == 0 && code != 0) {
    dev->inject_sync = code;
  } else if (kind == 1) {
    dev->inject_alloc = true;
  } else if (kind == 2 && (code == 1 || code == 2)) {
    ack::set_encode_stall_test(uint32_t(code));
  } else {
    set_error(format("ack_inject_fault: kind %d is not 0 (synchronisation, nonzero code), 1 (allocation) or 2 "
                     "(encode stall test, code 1 or 2)",
                     kind));
    return ACK_ERR_SHAPE;
  }
  return ACK_OK;
}

// ------------------------------------------------------------ vq4 entries --

ACK_EXPORT uint32_t ack_vq_schema(void) { return ACK_VQ_SCHEMA; }

ACK_EXPORT int32_t ack_kernel_manifest(char* out, size_t len, size_t* needed) {
  const size_t n = sizeof(kManifestJson);
  if (needed) *needed = n;
  if (!out) return needed ? ACK_OK : ACK_ERR_NULL;
  if (len < n) {
    set_error(format("kernel manifest needs %zu bytes, %zu given", n, len));
    return ACK_ERR_SIZE;
  }
  memcpy(out, kManifestJson, n);
  return ACK_OK;
}
ACK_EXPORT uint32_t ack_vq2_schema(void) { return ACK_VQ2_SCHEMA; }

namespace {

// Admission against live registry buffers, then enqueue. `handles` is in the
// plan's slot order (6 or 8 entries).
int32_t run_handles(const char* entry, const AckDevice* handle, const AckBuffer* const* handles,
                    const ack::Plan& plan) {
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  if (dev->poisoned) {
    set_error(format("%s: device poisoned by an earlier failed CUDA operation", entry));
    return ACK_ERR_POISONED;
  }
  const int n = plan.nslots();
  uint64_t caps[ack::kSlots] = {0}, ids[ack::kSlots] = {0};
  void* ptr[ack::kSlots] = {nullptr};
  for (int i = 0; i < n; ++i) {
    if (plan.schema == 2 && !handles[i] && !plan.required[i]) continue;  // an unused schema-2 slot
    BufferRec* b = nullptr;
    rc = buffer_of(*dev, handles[i], &b);
    if (rc) return rc;
    caps[i] = b->bytes;
    ids[i] = b->id;
    ptr[i] = b->ptr;
  }
  int slot = 0;
  ack::PlanError e = ack::validate_buffers(plan, caps, ids, &slot);
  if (e == ack::PlanError::None) {
    const std::array<uint32_t, 3> limits = {uint32_t(dev->prop.maxGridSize[0]), uint32_t(dev->prop.maxGridSize[1]),
                                            uint32_t(dev->prop.maxGridSize[2])};
    e = ack::validate_dispatch(plan, limits);
  }
  if (e != ack::PlanError::None) return plan_refused(entry, e, plan.schema, slot);
  DeviceScope scope(dev->ordinal);
  cudaError_t ce = ack::launch(plan, ptr, dev->stream);
  if (ce != cudaSuccess) return cuda_fail(*dev, ce, entry);
  return ACK_OK;
}

}  // namespace

ACK_EXPORT int32_t ack_vq(const AckDevice* dev, const AckBuffer* b0, const AckBuffer* b1, const AckBuffer* b2,
                          const AckBuffer* b3, const AckBuffer* out, const AckBuffer* status, const uint8_t* plan,
                          size_t plan_len) {
  if (!plan) {
    set_error("vq: null plan");
    return ACK_ERR_NULL;
  }
  if (plan_len != ACK_VQ_PUSH_BYTES) {
    set_error(format("vq: plan has %zu bytes, expected %u", plan_len, ACK_VQ_PUSH_BYTES));
    return ACK_ERR_SIZE;
  }
  ack::Plan p;
  ack::PlanError e = ack::parse_plan(plan, plan_len, &p);
  if (e != ack::PlanError::None) return plan_refused("vq", e, 1, 0);
  const AckBuffer* handles[6] = {b0, b1, b2, b3, out, status};
  return run_handles("vq", dev, handles, p);
}

ACK_EXPORT int32_t ack_vq2(const AckDevice* dev, const AckBuffer* const* slots, size_t nslots, const uint8_t* plan,
                           size_t plan_len) {
  if (!plan) {
    set_error("vq2: null plan");
    return ACK_ERR_NULL;
  }
  if (plan_len != ACK_VQ2_PLAN_BYTES) {
    set_error(format("vq2: plan has %zu bytes, expected %u", plan_len, ACK_VQ2_PLAN_BYTES));
    return ACK_ERR_SIZE;
  }
  if (!slots) {
    set_error("vq2: null slot array");
    return ACK_ERR_NULL;
  }
  if (nslots != ACK_VQ2_SLOTS) {
    set_error(format("vq2: %zu slots, expected %u", nslots, ACK_VQ2_SLOTS));
    return ACK_ERR_SIZE;
  }
  ack::Plan p;
  ack::PlanError e = ack::parse_plan(plan, plan_len, &p);
  if (e != ack::PlanError::None) return plan_refused("vq2", e, 2, 0);
  return run_handles("vq2", dev, slots, p);
}

// ---------------------------------------------- pipelined host-memory product --

namespace {

// Create the device's copy streams and events on first use.
cudaError_t pipeline_streams(Device& d) {
  cudaError_t e = cudaSuccess;
  if (!d.copy_in) e = cudaStreamCreateWithFlags(&d.copy_in, cudaStreamNonBlocking);
  if (e == cudaSuccess && !d.copy_out) e = cudaStreamCreateWithFlags(&d.copy_out, cudaStreamNonBlocking);
  for (cudaEvent_t& ev : d.ev)
    if (e == cudaSuccess && !ev) e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  return e;
}

// At least `bytes` of the device's pipeline scratch. Called with the device
// lock held and its streams idle (every call ends with a stream sync).
cudaError_t pipeline_scratch(Device& d, uint64_t bytes) {
  if (d.scratch_bytes >= bytes) return cudaSuccess;
  if (d.scratch) cudaFree(d.scratch);
  d.scratch = nullptr;
  d.scratch_bytes = 0;
  cudaError_t e = cudaMalloc(&d.scratch, bytes);
  if (e == cudaSuccess) d.scratch_bytes = bytes;
  return e;
}

}  // namespace

ACK_EXPORT int32_t ack_vq2_dense_host(const AckDevice* handle, const uint8_t* plan, size_t plan_len,
                                      const AckBuffer* codes, const AckBuffer* books, const float* x, float* y,
                                      uint32_t parts, uint32_t* status_out) {
  const char* entry = "vq2-dense-host";
  if (!plan || !x || !y || !status_out) {
    set_error(format("%s: null plan, host array or status pointer", entry));
    return ACK_ERR_NULL;
  }
  if (plan_len != ACK_VQ2_PLAN_BYTES) {
    set_error(format("%s: plan has %zu bytes, expected %u", entry, plan_len, ACK_VQ2_PLAN_BYTES));
    return ACK_ERR_SIZE;
  }
  ack::Plan p;
  ack::PlanError pe = ack::parse_plan(plan, plan_len, &p);
  if (pe != ack::PlanError::None) return plan_refused(entry, pe, 2, 0);
  if (p.op != ack::Op::Dense) {
    set_error(format("%s: the plan is not the dense product (op 16)", entry));
    return ACK_ERR_UNSUPPORTED_OP;
  }
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  if (dev->poisoned) {
    set_error(format("%s: device poisoned by an earlier failed CUDA operation", entry));
    return ACK_ERR_POISONED;
  }
  BufferRec *bc = nullptr, *bb = nullptr;
  if ((rc = buffer_of(*dev, codes, &bc)) || (rc = buffer_of(*dev, books, &bb))) return rc;
  // admission of the whole product: the host arrays stand in for in0 and out0
  // (their sizes are the caller's promise), the workspace for in4
  const uint64_t kHostX = ~uint64_t(0) - 1, kHostY = ~uint64_t(0) - 2, kWork = ~uint64_t(0) - 3,
                 kStatus = ~uint64_t(0) - 4;
  uint64_t caps[ack::kSlots] = {p.required[0], bc->bytes, bb->bytes, 0, p.required[4], p.required[5], 0, 4};
  uint64_t ids[ack::kSlots] = {kHostX, bc->id, bb->id, 0, p.required[4] ? kWork : 0, kHostY, 0, kStatus};
  int slot = 0;
  pe = ack::validate_buffers(p, caps, ids, &slot);
  if (pe != ack::PlanError::None) return plan_refused(entry, pe, 2, slot);
  const uint32_t E = p.batch;
  const uint64_t M = p.m, N = p.n, K = p.k;
  if (parts == 0) parts = uint32_t(std::min<uint64_t>(16, E));  // measured best for cfg2 M = 1 (12-24 alike)
  parts = uint32_t(std::min<uint64_t>(parts, E));
  const uint32_t per = (E + parts - 1) / parts;

  const uint64_t w_bytes = bc->bytes / E, book_bytes = bb->bytes / E;
  const uint64_t ws_part = (p.flags & 8u) ? ack::dense_tc_workspace_bytes(M, K, p.group, per) : 0;
  DeviceScope scope(dev->ordinal);
  cudaError_t e = pipeline_streams(*dev);
  if (e != cudaSuccess) return cuda_fail(*dev, e, entry);
  cudaStream_t cs = dev->stream, in = dev->copy_in, out = dev->copy_out;
  cudaEvent_t allocated = dev->ev[0], *h_done = dev->ev + 1, *k_done = dev->ev + 3, *d_done = dev->ev + 5;
  // scratch: all of X and Y (so no part waits for another's buffer), two
  // tensor-core workspaces (reused in stream order), the status word
  auto up = [](uint64_t v) { return (v + 255) & ~uint64_t(255); };
  const uint64_t x_all = uint64_t(E) * M * K * 4, y_all = uint64_t(E) * M * N * 4;
  const uint64_t need = up(x_all) + up(y_all) + 2 * up(ws_part) + 256;
  e = pipeline_scratch(*dev, need);
  if (e != cudaSuccess) return cuda_fail(*dev, e, entry);
  char* xd = static_cast<char*>(dev->scratch);
  char* yd = xd + up(x_all);
  void* wb[2] = {ws_part ? yd + up(y_all) : nullptr, ws_part ? yd + up(y_all) + up(ws_part) : nullptr};
  uint32_t* status = reinterpret_cast<uint32_t*>(static_cast<char*>(dev->scratch) + need - 256);
  auto fail = [&](cudaError_t err) { return cuda_fail(*dev, err, entry); };
  e = cudaMemsetAsync(status, 0, 4, cs);
  if (e == cudaSuccess) e = cudaEventRecord(allocated, cs);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(in, allocated, 0);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(out, allocated, 0);
  if (e != cudaSuccess) return fail(e);
  const char* xh = reinterpret_cast<const char*>(x);
  char* yh = reinterpret_cast<char*>(y);
  // the copies in run back to back on their stream; part c's product waits
  // only for its own X, its copy out only for its own product (each event is
  // waited on right after it is recorded, so one event of each kind serves
  // every part)
  for (uint32_t c = 0; c < parts && e == cudaSuccess; ++c) {
    const uint32_t e0 = c * per, ec = std::min<uint32_t>(per, E - std::min<uint32_t>(E, e0));
    if (!ec) break;
    const uint64_t xo = uint64_t(e0) * M * K * 4, yo = uint64_t(e0) * M * N * 4;
    e = cudaMemcpyAsync(xd + xo, xh + xo, uint64_t(ec) * M * K * 4, cudaMemcpyHostToDevice, in);
    if (e == cudaSuccess) e = cudaEventRecord(h_done[0], in);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, h_done[0], 0);
    if (e == cudaSuccess) {
      ack::Plan q = p;
      q.batch = ec;
      void* ptr[ack::kSlots] = {xd + xo, static_cast<char*>(bc->ptr) + uint64_t(e0) * w_bytes,
                                static_cast<char*>(bb->ptr) + uint64_t(e0) * book_bytes, nullptr, wb[c & 1u],
                                yd + yo, nullptr, status};
      e = ack::launch(q, ptr, cs);
    }
    if (e == cudaSuccess) e = cudaEventRecord(k_done[0], cs);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(out, k_done[0], 0);
    if (e == cudaSuccess) e = cudaMemcpyAsync(yh + yo, yd + yo, uint64_t(ec) * M * N * 4, cudaMemcpyDeviceToHost, out);
  }
  // the status word is read on the compute stream after the last copies out
  if (e == cudaSuccess) e = cudaEventRecord(d_done[0], out);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, d_done[0], 0);
  uint32_t host_status = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&host_status, status, 4, cudaMemcpyDeviceToHost, cs);
  if (e != cudaSuccess) return fail(e);
  e = sync_stream(*dev);
  if (e != cudaSuccess) return cuda_fail(*dev, e, entry);
  *status_out = host_status;
  return ACK_OK;
}

// ------------------------------------------------------ the NF4 comparator --
//
// nf4-decode/v1 and nf4-gemv/v1 (ffi.rs:7365 ack_nf4_decode, :8017
// ack_gemv_nf4; planners nf4_ops.rs:158-204 and :515-569): the same
// arguments, refusal names and return codes; the work is enqueued on the
// device's stream (ack_download waits for it), and `ms_out`, when given,
// reads NaN (no per-call duration is measured), as the reference reports a
// recorded dispatch.

namespace {

constexpr uint32_t kNf4Block = 64, kNf4NestedValues = 64 * 256, kNf4TableEntries = 16 + 256;

struct Nf4Operand {
  void* ptr;
  uint64_t bytes;
  uint64_t id;
};

uint64_t nf4_covered(uint64_t packed_bytes, uint64_t absmax_q_bytes, uint64_t absmax2_bytes) {
  return std::min({8 * (packed_bytes / 4), 4 * (absmax_q_bytes / 4) * kNf4Block,
                   (absmax2_bytes / 4) * kNf4NestedValues});
}

void no_duration(double* ms_out) {
  if (ms_out) *ms_out = std::nan("");
}

// Admission of one decode (nf4_ops.rs:158-204 and ffi.rs:7435-7490); on
// success fills `src` and returns ACK_OK.
int32_t nf4_decode_admit(const Nf4Operand* op, uint32_t n, uint32_t members, uint32_t selected,
                         uint32_t member_values, uint32_t src_base, uint32_t storage, ack::Nf4Source* src) {
  // op: packed, absmax_q, absmax2, tables, starts, offsets, ids, out
  const uint64_t covered = nf4_covered(op[0].bytes, op[1].bytes, op[2].bytes);
  const char* refused = nullptr;
  int32_t code = ACK_ERR_SHAPE;
  const uint32_t mv = selected == 0 ? 0 : member_values;
  if (n == 0) {
    refused = "nf4-zero-values";
  } else if (uint64_t(n) > (uint64_t(1) << 31)) {
    refused = "nf4-value-limit-exceeded";
    code = ACK_ERR_SIZE;
  } else if (members == 0) {
    refused = "nf4-members-out-of-range";
  } else if (selected != 0 && (mv == 0 || mv % kNf4Block != 0 || uint64_t(selected) * mv != n)) {
    refused = "nf4-selection-out-of-range";
  } else if (src_base % kNf4NestedValues != 0 || uint64_t(src_base) >= covered) {
    refused = "nf4-base-out-of-range";
  } else if (selected == 0 && n > std::min<uint64_t>(covered - src_base, 0xffffffffull)) {
    refused = "nf4-source-too-small";
    code = ACK_ERR_SIZE;
  }
  if (refused) {
    set_error(format("nf4-decode: %u values, %u member(s), %u selected, base %u, %llu covered: plan refused: %s", n,
                     members, selected, src_base, (unsigned long long)covered, refused));
    return code;
  }
  const uint64_t out_bytes = uint64_t(n) * (storage == 0 ? 4 : 2);
  struct Role {
    int slot;
    uint64_t needed;
    const char* name;
  } roles[] = {{3, 4ull * kNf4TableEntries, "tables"}, {4, 8ull * members, "starts"}, {5, 4ull * members, "offsets"},
               {6, 8ull * selected, "ids"}, {7, out_bytes, "output"}};
  for (const Role& r : roles) {
    if (r.slot == 6 && selected == 0) continue;
    if (op[r.slot].bytes < r.needed) {
      set_error(format("nf4-decode: %s of %llu bytes for %llu: plan refused: nf4-%s-too-small", r.name,
                       (unsigned long long)op[r.slot].bytes, (unsigned long long)r.needed, r.name));
      return ACK_ERR_SIZE;
    }
  }
  for (int i = 0; i < 7; ++i) {
    if (i == 6 && selected == 0) continue;
    if (op[i].id == op[7].id) {
      set_error("nf4-decode: plan refused: nf4-output-aliases-input");
      return ACK_ERR_SHAPE;
    }
  }
  *src = ack::Nf4Source{static_cast<const uint32_t*>(op[0].ptr), static_cast<const uint32_t*>(op[1].ptr),
                        static_cast<const float*>(op[2].ptr), static_cast<const float*>(op[3].ptr),
                        static_cast<const uint32_t*>(op[4].ptr), static_cast<const float*>(op[5].ptr), members,
                        src_base, uint32_t(std::min<uint64_t>(covered - src_base, 0xffffffffull))};
  return ACK_OK;
}

// Admission of one grouped GEMV (nf4_ops.rs:515-569 and ffi.rs:8080-8145).
int32_t nf4_gemv_admit(const Nf4Operand* op, uint32_t rows, uint32_t max_rows, uint32_t n, uint32_t k,
                       uint32_t lda, uint32_t groups, uint32_t members, uint32_t src_base, ack::Nf4Gemv* g) {
  // op: a, packed, absmax_q, absmax2, tables, starts, offsets, groups_table, c
  const uint64_t covered = nf4_covered(op[1].bytes, op[2].bytes, op[3].bytes);
  const char* refused = nullptr;
  int32_t code = ACK_ERR_SHAPE;
  const uint32_t pitch = lda == 0 ? k : lda;
  const uint64_t weight = uint64_t(n) * k, limit = 0xffffffffull;
  if (rows == 0 || max_rows == 0 || n == 0 || k == 0) {
    refused = "nf4-matmul-zero-extent";
  } else if (groups == 0 || groups > 65535u) {
    refused = "nf4-matmul-groups-out-of-range";
  } else if (max_rows > rows) {
    refused = "nf4-matmul-rows-out-of-range";
  } else if (max_rows > 16u) {
    refused = "nf4-gemv-rows-above-16";
  } else if (k % 8u) {
    refused = "nf4-matmul-row-not-whole-words";
  } else if (pitch < k) {
    refused = "nf4-matmul-pitch-below-width";
  } else if (pitch % 8u) {
    refused = "nf4-gemv-pitch-not-whole-words";
  } else if (members == 0) {
    refused = "nf4-members-out-of-range";
  } else if (src_base % kNf4NestedValues != 0 || uint64_t(src_base) >= covered) {
    refused = "nf4-base-out-of-range";
  } else if (weight > covered - src_base) {
    refused = "nf4-source-too-small";
    code = ACK_ERR_SIZE;
  } else if (uint64_t(rows - 1) * pitch + k > limit || uint64_t(rows) * n > limit || weight > limit) {
    refused = "nf4-matmul-address-limit-exceeded";
    code = ACK_ERR_SIZE;
  }
  if (refused) {
    set_error(format("nf4-gemv: %u group(s), %u rows (largest %u) x %u x %u, base %u, %llu covered: plan refused: %s",
                     groups, rows, max_rows, n, k, src_base, (unsigned long long)covered, refused));
    return code;
  }
  const uint64_t a_elements = uint64_t(rows - 1) * pitch + k;
  struct Role {
    int slot;
    uint64_t needed;
    const char* name;
  } roles[] = {{0, 2 * a_elements, "a"}, {4, 4ull * kNf4TableEntries, "tables"}, {5, 8ull * members, "starts"},
               {6, 4ull * members, "offsets"}, {7, 12ull * groups, "groups"}, {8, 4ull * rows * n, "output"}};
  for (const Role& r : roles)
    if (op[r.slot].bytes < r.needed) {
      set_error(format("nf4-gemv: %s of %llu bytes for %llu: plan refused: nf4-matmul-%s-too-small", r.name,
                       (unsigned long long)op[r.slot].bytes, (unsigned long long)r.needed, r.name));
      return ACK_ERR_SIZE;
    }
  for (int i = 0; i < 8; ++i)
    if (op[i].id == op[8].id) {
      set_error("nf4-gemv: plan refused: nf4-matmul-output-aliases-input");
      return ACK_ERR_SHAPE;
    }
  const uint32_t src_limit = uint32_t(std::min<uint64_t>(covered - src_base, limit - src_base));
  *g = ack::Nf4Gemv{static_cast<const uint4*>(op[0].ptr), static_cast<float*>(op[8].ptr),
                    static_cast<const uint32_t*>(op[7].ptr), n, k, pitch, rows, groups,
                    ack::Nf4Source{static_cast<const uint32_t*>(op[1].ptr), static_cast<const uint32_t*>(op[2].ptr),
                                   static_cast<const float*>(op[3].ptr), static_cast<const float*>(op[4].ptr),
                                   static_cast<const uint32_t*>(op[5].ptr), static_cast<const float*>(op[6].ptr),
                                   members, src_base, src_limit}};
  return ACK_OK;
}

// The handle entries' common part: resolve `count` handles (null allowed
// where `optional` says so) against the locked device.
int32_t nf4_resolve(Device& d, const AckBuffer* const* handles, int count, uint64_t optional_mask,
                    Nf4Operand* out) {
  for (int i = 0; i < count; ++i) {
    if (!handles[i] && ((optional_mask >> i) & 1u)) {
      out[i] = Nf4Operand{nullptr, 0, ~uint64_t(0) - uint64_t(i)};
      continue;
    }
    BufferRec* b = nullptr;
    const int32_t rc = buffer_of(d, handles[i], &b);
    if (rc) return rc;
    out[i] = Nf4Operand{b->ptr, b->bytes, b->id};
  }
  return ACK_OK;
}

}  // namespace

ACK_EXPORT int32_t ack_nf4_decode(const AckDevice* handle, const AckBuffer* packed, const AckBuffer* absmax_q,
                                  const AckBuffer* absmax2, const AckBuffer* tables, const AckBuffer* starts,
                                  const AckBuffer* offsets, const AckBuffer* ids, const AckBuffer* out, uint32_t n,
                                  uint32_t members, uint32_t selected, uint32_t member_values, uint32_t src_base,
                                  uint32_t storage, double* ms_out) {
  no_duration(ms_out);
  if (storage > 2) {
    set_error("nf4-decode: plan refused: nf4-storage-out-of-range");
    return ACK_ERR_SHAPE;
  }
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  if ((rc = refuse_poisoned(*dev, "nf4-decode"))) return rc;
  const AckBuffer* hs[8] = {packed, absmax_q, absmax2, tables, starts, offsets, ids, out};
  Nf4Operand op[8];
  // the whole-source decode reads no ids
  if ((rc = nf4_resolve(*dev, hs, 8, selected == 0 ? (1u << 6) : 0u, op))) return rc;
  ack::Nf4Source src;
  if ((rc = nf4_decode_admit(op, n, members, selected, member_values, src_base, storage, &src))) return rc;
  DeviceScope scope(dev->ordinal);
  const cudaError_t e = ack::nf4_decode(src, static_cast<const uint32_t*>(op[6].ptr), op[7].ptr, n, selected,
                                        member_values, storage, dev->stream);
  return e == cudaSuccess ? ACK_OK : cuda_fail(*dev, e, "nf4-decode");
}

ACK_EXPORT int32_t ack_gemv_nf4(const AckDevice* handle, const AckBuffer* a, const AckBuffer* packed,
                                const AckBuffer* absmax_q, const AckBuffer* absmax2, const AckBuffer* tables,
                                const AckBuffer* starts, const AckBuffer* offsets, const AckBuffer* groups_table,
                                const AckBuffer* c, uint32_t rows, uint32_t max_rows, uint32_t n, uint32_t k,
                                uint32_t lda, uint32_t groups, uint32_t members, uint32_t src_base, uint32_t elem,
                                double* ms_out) {
  no_duration(ms_out);
  if (elem > 1) {
    set_error("nf4-gemv: plan refused: nf4-matmul-elem-out-of-range");
    return ACK_ERR_SHAPE;
  }
  std::shared_ptr<Device> dev;
  int32_t rc = lookup(handle, &dev);
  if (rc) return rc;
  std::unique_lock<std::mutex> lk;
  rc = acquire(*dev, &lk);
  if (rc) return rc;
  if ((rc = refuse_poisoned(*dev, "nf4-gemv"))) return rc;
  const AckBuffer* hs[9] = {a, packed, absmax_q, absmax2, tables, starts, offsets, groups_table, c};
  Nf4Operand op[9];
  if ((rc = nf4_resolve(*dev, hs, 9, 0, op))) return rc;
  ack::Nf4Gemv g;
  if ((rc = nf4_gemv_admit(op, rows, max_rows, n, k, lda, groups, members, src_base, &g))) return rc;
  DeviceScope scope(dev->ordinal);
  const cudaError_t e = ack::nf4_gemv(g, max_rows, elem, dev->stream);
  return e == cudaSuccess ? ACK_OK : cuda_fail(*dev, e, "nf4-gemv");
}

// Device-pointer forms (no counterpart in the reference) for callers whose
// data is in device memory already (PyTorch tensors): the same admission;
// `ptrs` / `bytes` in the handle entries' argument order, work enqueued on
// `stream` on the current device. Operands are told apart by address.
ACK_EXPORT int32_t ack_nf4_decode_launch(void* const* ptrs, const uint64_t* bytes, uint32_t n, uint32_t members,
                                         uint32_t selected, uint32_t member_values, uint32_t src_base,
                                         uint32_t storage, void* stream) {
  if (!ptrs || !bytes) return ACK_ERR_NULL;
  if (storage > 2) {
    set_error("nf4-decode: plan refused: nf4-storage-out-of-range");
    return ACK_ERR_SHAPE;
  }
  Nf4Operand op[8];
  for (int i = 0; i < 8; ++i) {
    if (!ptrs[i] && !(i == 6 && selected == 0)) {
      set_error(format("nf4-decode: operand %d is null", i));
      return ACK_ERR_NULL;
    }
    op[i] = Nf4Operand{ptrs[i], bytes[i], ptrs[i] ? uint64_t(reinterpret_cast<uintptr_t>(ptrs[i])) : ~uint64_t(0)};
  }
  ack::Nf4Source src;
  const int32_t rc = nf4_decode_admit(op, n, members, selected, member_values, src_base, storage, &src);
  if (rc) return rc;
  const cudaError_t e = ack::nf4_decode(src, static_cast<const uint32_t*>(op[6].ptr), op[7].ptr, n, selected,
                                        member_values, storage, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error(format("nf4-decode: %s", cudaGetErrorString(e)));
    return ACK_ERR_VULKAN;
  }
  return ACK_OK;
}

ACK_EXPORT int32_t ack_gemv_nf4_launch(void* const* ptrs, const uint64_t* bytes, uint32_t rows, uint32_t max_rows,
                                       uint32_t n, uint32_t k, uint32_t lda, uint32_t groups, uint32_t members,
                                       uint32_t src_base, uint32_t elem, void* stream) {
  if (!ptrs || !bytes) return ACK_ERR_NULL;
  if (elem > 1) {
    set_error("nf4-gemv: plan refused: nf4-matmul-elem-out-of-range");
    return ACK_ERR_SHAPE;
  }
  Nf4Operand op[9];
  for (int i = 0; i < 9; ++i) {
    if (!ptrs[i]) {
      set_error(format("nf4-gemv: operand %d is null", i));
      return ACK_ERR_NULL;
    }
    op[i] = Nf4Operand{ptrs[i], bytes[i], uint64_t(reinterpret_cast<uintptr_t>(ptrs[i]))};
  }
  ack::Nf4Gemv g;
  const int32_t rc = nf4_gemv_admit(op, rows, max_rows, n, k, lda, groups, members, src_base, &g);
  if (rc) return rc;
  const cudaError_t e = ack::nf4_gemv(g, max_rows, elem, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error(format("nf4-gemv: %s", cudaGetErrorString(e)));
    return ACK_ERR_VULKAN;
  }
  return ACK_OK;
}

namespace {
int32_t launch_ptrs(const uint8_t* plan, size_t plan_len, const AckVqOperands* ops, void* stream,
                    const ack::PeerY* peers);
}  // namespace

ACK_EXPORT int32_t ack_vq_launch(const uint8_t* plan, size_t plan_len, const AckVqOperands* ops, void* stream) {
  return launch_ptrs(plan, plan_len, ops, stream, nullptr);
}

// ack_vq_launch's op-16 plan (M = 1, W stored N x K, canonical) whose outputs
// are also written into `npeers` other ranks' output slots (`peers`: device
// pointers valid here, e.g. CUDA IPC mappings), at Y's offsets.
ACK_EXPORT int32_t ack_vq_dense_peers(const uint8_t* plan, size_t plan_len, const AckVqOperands* ops,
                                      float* const* peers, uint32_t npeers, void* stream) {
  if (npeers > ack::kMaxPeers || (npeers && !peers)) {
    set_error(format("vq2-dense-peers: %u peer slots (at most %u)", npeers, ack::kMaxPeers));
    return ACK_ERR_SHAPE;
  }
  ack::PeerY py{};
  for (uint32_t i = 0; i < npeers; ++i) {
    if (!peers[i]) {
      set_error(format("vq2-dense-peers: peer slot %u is null", i));
      return ACK_ERR_NULL;
    }
    py.dst[i] = peers[i];
  }
  py.n = npeers;
  return launch_ptrs(plan, plan_len, ops, stream, &py);
}

// Step flags of the peer-store products: publish this rank's epoch into every
// rank's flag array, and wait (bounded) for every rank's epoch here.
ACK_EXPORT int32_t ack_peer_signal(uint32_t* const* flags, uint32_t world, uint32_t rank, uint32_t epoch,
                                   void* stream) {
  if (!flags) return ACK_ERR_NULL;
  const cudaError_t e = ack::peer_signal(flags, world, rank, epoch, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error(format("peer-signal: %s", cudaGetErrorString(e)));
    return e == cudaErrorInvalidValue ? ACK_ERR_SHAPE : ACK_ERR_VULKAN;
  }
  return ACK_OK;
}

ACK_EXPORT int32_t ack_peer_wait(const uint32_t* flags, uint32_t world, uint32_t epoch, uint32_t* status,
                                 uint32_t polls, void* stream) {
  if (!flags || !status) return ACK_ERR_NULL;
  const cudaError_t e = ack::peer_wait(flags, world, epoch, status, polls ? polls : (1u << 24),
                                       static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_error(format("peer-wait: %s", cudaGetErrorString(e)));
    return e == cudaErrorInvalidValue ? ACK_ERR_SHAPE : ACK_ERR_VULKAN;
  }
  return ACK_OK;
}

// Device memory another process can map (CUDA IPC, no multicast object):
// allocate zeroed on the current device and write its 64-byte handle.
ACK_EXPORT int32_t ack_peer_alloc(uint64_t bytes, void** ptr, uint8_t* handle) {
  if (!ptr || !handle) return ACK_ERR_NULL;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    if (p) cudaFree(p);
    cudaGetLastError();
    set_error(format("peer-alloc of %llu bytes: %s", (unsigned long long)bytes, cudaGetErrorString(e)));
    return ACK_ERR_VULKAN;
  }
  static_assert(sizeof(h) == 64, "a CUDA IPC memory handle is 64 bytes");
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return ACK_OK;
}

ACK_EXPORT int32_t ack_peer_open(const uint8_t* handle, void** ptr) {
  if (!ptr || !handle) return ACK_ERR_NULL;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    set_error(format("peer-open: %s", cudaGetErrorString(e)));
    return ACK_ERR_VULKAN;
  }
  return ACK_OK;
}

ACK_EXPORT int32_t ack_peer_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? ACK_OK : ACK_ERR_VULKAN;
}

ACK_EXPORT int32_t ack_peer_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? ACK_OK : ACK_ERR_VULKAN;
}

namespace {
int32_t launch_ptrs(const uint8_t* plan, size_t plan_len, const AckVqOperands* ops, void* stream,
                    const ack::PeerY* peers) {
  if (!plan || !ops) {
    set_error(!plan ? "vq: null plan" : "vq: null operands");
    return ACK_ERR_NULL;
  }
  if (ops->size < sizeof(AckVqOperands)) {
    set_error(format("AckVqOperands of %u bytes is smaller than this library's %zu", ops->size,
                     sizeof(AckVqOperands)));
    return ACK_ERR_ABI;
  }
  if (plan_len != ACK_VQ_PUSH_BYTES && plan_len != ACK_VQ2_PLAN_BYTES) {
    set_error(format("vq: plan has %zu bytes, expected %u or %u", plan_len, ACK_VQ_PUSH_BYTES, ACK_VQ2_PLAN_BYTES));
    return ACK_ERR_SIZE;
  }
  const char* entry = plan_len == ACK_VQ_PUSH_BYTES ? "vq" : "vq2";
  ack::Plan p;
  ack::PlanError e = ack::parse_plan(plan, plan_len, &p);
  if (e != ack::PlanError::None) return plan_refused(entry, e, p.schema, 0);
  const int n = p.nslots();
  if (ops->nslots != uint32_t(n)) {
    set_error(format("%s: %u operand slots, expected %d", entry, ops->nslots, n));
    return ACK_ERR_SIZE;
  }
  uint64_t ids[ack::kSlots] = {0}, caps[ack::kSlots] = {0};
  void* ptr[ack::kSlots] = {nullptr};
  for (int i = 0; i < n; ++i) {
    ptr[i] = ops->ptr[i];
    ids[i] = uint64_t(reinterpret_cast<uintptr_t>(ops->ptr[i]));
    caps[i] = ops->bytes[i];
  }
  int slot = 0;
  e = ack::validate_buffers(p, caps, ids, &slot);
  if (e != ack::PlanError::None) return plan_refused(entry, e, p.schema, slot);
  // pointers: 4-byte aligned; written ranges disjoint from every other used range
  for (int i = 0; i < n; ++i)
    if (p.required[i] && (ids[i] & 3u)) return plan_refused(entry, ack::PlanError::Misaligned, 2, i);
  const int first_out = p.first_output();
  // the fit's workspace (in4) is written too
  const int first_written = p.writes_in4() ? 4 : first_out;
  for (int o = first_written; o < n; ++o) {
    if (!p.required[o]) continue;
    for (int i = 0; i < n; ++i) {
      if (i == o || !p.required[i]) continue;
      const uint64_t a0 = ids[o], a1 = ids[o] + p.required[o], b0 = ids[i], b1 = ids[i] + p.required[i];
      if (a0 < b1 && b0 < a1) {
        const bool status = o == p.status_slot() || i == p.status_slot();
        return plan_refused(entry, status ? ack::PlanError::StatusAlias : ack::PlanError::OutputAlias, p.schema, 0);
      }
    }
  }
  cudaError_t ce = peers ? ack::dense_peers(p, ptr, *peers, static_cast<cudaStream_t>(stream))
                        : ack::launch(p, ptr, static_cast<cudaStream_t>(stream));
  if (ce == cudaErrorNotSupported && peers) {
    set_error(format("%s: the peer-store product takes op 16 with M = 1, W stored N x K, canonical codes, "
                     "K a multiple of 256 g and enough rows for the byte-pair kernel", entry));
    return ACK_ERR_UNSUPPORTED_OP;
  }
  if (ce != cudaSuccess) {
    set_error(format("%s: launch: %s (%s)", entry, cudaGetErrorName(ce), cudaGetErrorString(ce)));
    return ACK_ERR_VULKAN;
  }
  return ACK_OK;
}
}  // namespace

// ---------------------------------------------- encode without allocation --
// For callers that may not allocate device memory themselves or through this
// library: the caller passes device pointers to x, the books, the codes and
// a cleared status word; the only scratch is the library's static array.

ACK_EXPORT int32_t ack_vq_encode_noalloc(const float* x, uint64_t count, uint32_t batch, const float* books,
                                         uint32_t group, uint32_t* codes, uint32_t* status, void* stream) {
  const char* entry = "vq-encode-noalloc";
  if (!x || !books || !codes || !status) {
    set_error(format("%s: null pointer", entry));
    return ACK_ERR_NULL;
  }
  if (group != 8 && group != 16 && group != 32) {
    set_error(format("%s: group %u is not 8, 16 or 32", entry, group));
    return ACK_ERR_SHAPE;
  }
  if (count == 0 || count > (uint64_t(1) << 40)) {
    set_error(format("%s: %llu values per tensor (1 to 2^40 accepted)", entry, (unsigned long long)count));
    return ACK_ERR_SHAPE;
  }
  if (batch == 0 || batch > ack::kStaticEncodeBooks) {
    set_error(format("%s: batch of %u tensors exceeds the %u books its static scratch holds", entry, batch,
                     ack::kStaticEncodeBooks));
    return ACK_ERR_SIZE;
  }
  const uintptr_t px = reinterpret_cast<uintptr_t>(x), pb = reinterpret_cast<uintptr_t>(books),
                  pc = reinterpret_cast<uintptr_t>(codes), ps = reinterpret_cast<uintptr_t>(status);
  if ((px | pb | pc | ps) & 3u) {
    set_error(format("%s: pointers must be 4-byte aligned", entry));
    return ACK_ERR_SHAPE;
  }
  // written ranges (codes, status) disjoint from every other range
  const uint64_t words = ack::packed_words(count, group);
  const uint64_t rx[2] = {px, px + uint64_t(batch) * count * 4}, rb[2] = {pb, pb + uint64_t(batch) * 16 * group * 4};
  const uint64_t rc[2] = {pc, pc + uint64_t(batch) * words * 4}, rs[2] = {ps, ps + 4};
  auto overlap = [](const uint64_t* a, const uint64_t* b) { return a[0] < b[1] && b[0] < a[1]; };
  if (overlap(rc, rx) || overlap(rc, rb) || overlap(rc, rs) || overlap(rs, rx) || overlap(rs, rb)) {
    set_error(format("%s: the codes or the status word overlap another operand", entry));
    return ACK_ERR_SHAPE;
  }
  cudaError_t ce = ack::encode_noalloc(x, count, batch, books, group, codes, status, static_cast<cudaStream_t>(stream));
  if (ce != cudaSuccess) {
    set_error(format("%s: launch: %s (%s)", entry, cudaGetErrorName(ce), cudaGetErrorString(ce)));
    return ACK_ERR_VULKAN;
  }
  return ACK_OK;
}

// ------------------------------------------------------- planner probes --

ACK_EXPORT int32_t ack_vq_plan_probe(const uint8_t* plan, size_t plan_len, uint64_t required_bytes[8],
                                     uint32_t* work_items, uint32_t dispatch[3]) {
  if (!plan) {
    set_error("vq: null plan");
    return ACK_ERR_NULL;
  }
  if (plan_len != ACK_VQ_PUSH_BYTES && plan_len != ACK_VQ2_PLAN_BYTES) {
    set_error(format("vq: plan has %zu bytes, expected %u", plan_len, ACK_VQ_PUSH_BYTES));
    return ACK_ERR_SIZE;
  }
  ack::Plan p;
  ack::PlanError e = ack::parse_plan(plan, plan_len, &p);
  if (e != ack::PlanError::None) return plan_refused(p.schema == 1 ? "vq" : "vq2", e, p.schema, 0);
  if (required_bytes)
    for (int i = 0; i < 8; ++i) required_bytes[i] = p.required[i];
  if (work_items) *work_items = p.work_items;
  if (dispatch)
    for (int i = 0; i < 3; ++i) dispatch[i] = p.dispatch[i];
  return ACK_OK;
}

ACK_EXPORT int32_t ack_vq_plan_validate_buffers(const uint8_t* plan, size_t plan_len, const uint64_t* capacities,
                                                const uint64_t* ids, size_t n) {
  if (!plan || !capacities || !ids) return ACK_ERR_NULL;
  ack::Plan p;
  if (plan_len != ACK_VQ_PUSH_BYTES && plan_len != ACK_VQ2_PLAN_BYTES) return ACK_ERR_SIZE;
  ack::PlanError e = ack::parse_plan(plan, plan_len, &p);
  if (e != ack::PlanError::None) return plan_refused("vq", e, p.schema, 0);
  if (n != size_t(p.nslots())) {
    set_error(format("vq: %zu slots, expected %d", n, p.nslots()));
    return ACK_ERR_SIZE;
  }
  int slot = 0;
  e = ack::validate_buffers(p, capacities, ids, &slot);
  if (e != ack::PlanError::None) return plan_refused(p.schema == 1 ? "vq" : "vq2", e, p.schema, slot);
  return ACK_OK;
}

ACK_EXPORT int32_t ack_vq_plan_validate_dispatch(const uint8_t* plan, size_t plan_len, const uint32_t limits[3]) {
  if (!plan || !limits) return ACK_ERR_NULL;
  ack::Plan p;
  if (plan_len != ACK_VQ_PUSH_BYTES && plan_len != ACK_VQ2_PLAN_BYTES) return ACK_ERR_SIZE;
  ack::PlanError e = ack::parse_plan(plan, plan_len, &p);
  if (e != ack::PlanError::None) return plan_refused("vq", e, p.schema, 0);
  e = ack::validate_dispatch(p, {limits[0], limits[1], limits[2]});
  if (e != ack::PlanError::None) return plan_refused(p.schema == 1 ? "vq" : "vq2", e, p.schema, 0);
  return ACK_OK;
}

// noalloc.cu -- dg_pkm_forward_noalloc: the PKM sequence forward with its
// scratch taken from a fixed device array, so the call allocates nothing.
//
// Who needs it: a caller that may not allocate device memory while it runs the
// recurrence -- a serving loop whose memory is sized and reserved up front and
// must not grow or fragment between requests, code that runs inside a host
// callback or under a memory manager that forbids allocation, or a step that
// has to take the same memory on every call.  dg_pkm_forward allocates its
// scratch from the stream-ordered pool when the caller hands it none; this
// entry point never does.
//
// The only scratch any PKM kernel here uses is the warp-specialised kernel's
// per-row hazard codes (B*H*T*64 int16, written in full by its pre-pass before
// they are read, so nothing in the array has to start at zero).  The array is a
// file-scope __device__ object of kNoAllocBytes.  Set-up: every call made outside
// stream capture, with the device current, looks up the array's address there
// (cudaGetSymbolAddress, return code checked; cheap once the module is loaded) and
// caches it per device; a call made while its stream is capturing uses the cached
// address, so the first call on a device should come before any stream capture.
// Looking the address up again outside capture means that a device reset, which can
// reload the module at another address, leaves no stale address behind for later
// uncaptured calls.  Calls whose scratch need exceeds the array are rejected with
// DG_ERR_WORKSPACE before any launch.
// Calls that overlap in time on one device share the array and race: the
// caller serializes them (one stream, or events between streams).
#include <mutex>

#include "dg_common.cuh"

namespace {

constexpr size_t kNoAllocBytes = size_t(16) << 20;        // 16 MiB: B*H*T up to 131072
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_mu;
void* g_addr[kMaxDevices];       // device address of g_noalloc_scratch per device, set once
bool g_addr_set[kMaxDevices];

// address of the scratch array on the current device: looked up on every call outside
// stream capture, taken from the per-device cache under capture
int scratch_address(cudaStream_t stream, void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    if (dev < 0 || dev >= kMaxDevices) return DG_ERR_UNSUPPORTED;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &cs);
    if (e != cudaSuccess) return dg_host::record_cuda_error(e);
    std::lock_guard<std::mutex> lock(g_mu);
    if (cs == cudaStreamCaptureStatusNone || !g_addr_set[dev]) {
        void* a = nullptr;
        e = cudaGetSymbolAddress(&a, g_noalloc_scratch);
        if (e != cudaSuccess) return dg_host::record_cuda_error(e);
        g_addr[dev] = a;
        g_addr_set[dev] = true;
    }
    *out = g_addr[dev];
    return DG_OK;
}

}  // namespace

extern "C" {

size_t dg_pkm_forward_workspace_size(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                                     int algo);
int dg_pkm_forward_ex(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh, const void* v,
                      const void* beta, const void* wk, const void* wq, const int64_t* idx, const void* decay,
                      int dynamic_decay, void* state, void* out, void* saved_s_act, int32_t* dev_status, int algo,
                      void* workspace, size_t workspace_bytes, void* stream);

int dg_pkm_forward_noalloc(int dtype, int B, int H, int T, int active, int64_t total_slots, int dh,
                           const void* v, const void* beta, const void* wk, const void* wq, const int64_t* idx,
                           const void* decay, int dynamic_decay, void* state, void* out, void* saved_s_act,
                           int32_t* dev_status, void* stream) {
    const size_t need = dg_pkm_forward_workspace_size(dtype, B, H, T, active, total_slots, dh, DG_PKM_AUTO);
    if (need > kNoAllocBytes) return DG_ERR_WORKSPACE;
    // the look-up runs whether or not this call needs scratch, so that the cache is set
    // before any call made under capture
    void* addr = nullptr;
    const int rc = scratch_address(static_cast<cudaStream_t>(stream), &addr);
    if (rc != DG_OK) return rc;
    void* ws = need ? addr : nullptr;
    return dg_pkm_forward_ex(dtype, B, H, T, active, total_slots, dh, v, beta, wk, wq, idx, decay, dynamic_decay,
                             state, out, saved_s_act, dev_status, DG_PKM_AUTO, ws, ws ? kNoAllocBytes : 0, stream);
}

}  // extern "C"

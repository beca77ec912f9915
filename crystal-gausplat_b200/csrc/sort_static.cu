// sort_static.cu — gsc_sort_pairs_u64_static: the stable (u64 key, u32 value)
// radix sort of gsc_sort_pairs_u64, for callers that cannot allocate device
// memory.
//
// Who needs it: code that runs where cudaMalloc is off limits or unsafe -- a
// host that hands every device byte to its own pool allocator and forbids
// side allocations, a real-time or plugin thread that must not take the
// driver's allocation locks, or a caller that has no gsc_ctx (creating one
// allocates). Such a caller passes its keys, values and a stream; everything
// else the sort needs lives in one fixed device array defined below.
//
// Limits and rules:
//  - The scratch is a file-scope __device__ array of kStaticScratchBytes
//    (about 3.7 MB). Every GPU on which the library's device code is loaded
//    holds it until the process exits. With CUDA's lazy module loading (the
//    default since CUDA 12.2) that load, and so the reservation of the
//    array, may happen only at the first call on a device: make that first
//    call during initialisation, outside real-time threads and outside any
//    stream capture.
//  - n may be at most GSC_STATIC_SORT_MAX_PAIRS (262144); larger sizes are
//    rejected with GSC_ERR_INVALID before any GPU work is queued.
//  - The first call on a device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current) and caches it for the
//    life of the process, so cudaDeviceReset (or destroying the primary
//    context) is not supported while the library is in use.
//  - Device-side errors (a look-back wait that gave up, a bounds check) land
//    in an error word at the end of the array; the next call clears it.
//    gsc_sort_pairs_u64_static_status(stream) waits for the stream, reads
//    and clears the word and reports it, without allocating.
//  - All calls share the one array, and each call clears the parts that must
//    start at zero (histograms, look-back flags, tickets) on its stream.
//    Calls whose GPU work overlaps -- on two streams, or from two threads --
//    race on the array; serialise them.
//  - No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"

namespace gs {
namespace {

constexpr int64_t kMaxPairs = GSC_STATIC_SORT_MAX_PAIRS;
constexpr int kMaxDevices = 64;

constexpr size_t a256(size_t x) { return (x + 255) & ~(size_t)255; }
// Same layout as the context-scratch sort: alternate keys, alternate values,
// then histograms + look-back status + tickets for up to 8 passes.
constexpr size_t kSortBytes = a256((size_t)kMaxPairs * 8) + a256((size_t)kMaxPairs * 4) +
                              a256(8 * 256 * 4 + 8 * (size_t)((kMaxPairs + 4095) / 4096) * 256 * 4 + 8 * 4);
constexpr size_t kStaticScratchBytes = kSortBytes + 256;  // + device error word

}  // namespace

// The scratch array. Host code must not pass `g_static_sort_scratch` to a
// kernel: on the host that name is only a stand-in, not a device address.
static __device__ __align__(256) unsigned char g_static_sort_scratch[kStaticScratchBytes];

namespace {

std::mutex g_mu;
void* g_addr[kMaxDevices] = {};

int scratch_address(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_addr[device]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_sort_scratch);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_static_sort_scratch)");
    g_addr[device] = p;
  }
  *out = g_addr[device];
  return GSC_OK;
}

}  // namespace
}  // namespace gs

using namespace gs;

extern "C" GSC_API int gsc_sort_pairs_u64_static(uint64_t* keys, uint32_t* values, int64_t n,
                                                 int begin_bit, int end_bit, void* stream) {
  GS_REQUIRE(n >= 0, "gsc_sort_pairs_u64_static: n must be >= 0");
  if (n > GSC_STATIC_SORT_MAX_PAIRS) {
    set_error("gsc_sort_pairs_u64_static: n = " + std::to_string(n) + " exceeds the fixed scratch limit of " +
              std::to_string((long long)GSC_STATIC_SORT_MAX_PAIRS) + " pairs; use gsc_sort_pairs_u64");
    return GSC_ERR_INVALID;
  }
  GS_REQUIRE(begin_bit >= 0 && end_bit <= 64 && begin_bit <= end_bit,
             "gsc_sort_pairs_u64_static: bad bit range");
  if (n <= 1 || begin_bit == end_bit) return GSC_OK;
  GS_REQUIRE(keys && values, "gsc_sort_pairs_u64_static: null keys/values");
  int device = 0;
  GS_CK(cudaGetDevice(&device));
  GS_REQUIRE(device >= 0 && device < kMaxDevices, "gsc_sort_pairs_u64_static: device index too large");
  void* base = nullptr;
  int rc = scratch_address(device, &base);
  if (rc != GSC_OK) return rc;
  if (sort_scratch_bytes(n, begin_bit, end_bit) > kSortBytes) {
    set_error("gsc_sort_pairs_u64_static: internal scratch layout exceeds the fixed array");
    return GSC_ERR_INVALID;
  }
  // A stack context carrying only what the sort launcher reads: the stream,
  // the SM count and the error word (the last 256 bytes of the array).
  gsc_ctx c;
  c.device = device;
  c.stream = (cudaStream_t)stream;
  GS_CK(cudaDeviceGetAttribute(&c.num_sms, cudaDevAttrMultiProcessorCount, device));
  c.err = reinterpret_cast<uint32_t*>(static_cast<char*>(base) + kSortBytes);
  GS_CK(cudaMemsetAsync(c.err, 0, 4, c.stream));
  return launch_sort_pairs(&c, keys, values, n, begin_bit, end_bit, static_cast<char*>(base));
}

extern "C" GSC_API int gsc_sort_pairs_u64_static_status(void* stream) {
  int device = 0;
  GS_CK(cudaGetDevice(&device));
  GS_REQUIRE(device >= 0 && device < kMaxDevices, "gsc_sort_pairs_u64_static_status: device index too large");
  void* base = nullptr;
  int rc = scratch_address(device, &base);
  if (rc != GSC_OK) return rc;
  uint32_t* err = reinterpret_cast<uint32_t*>(static_cast<char*>(base) + kSortBytes);
  cudaStream_t s = (cudaStream_t)stream;
  uint32_t flags = 0;  // pageable host word: the copy completes before the call returns
  GS_CK(cudaStreamSynchronize(s));
  GS_CK(cudaMemcpyAsync(&flags, err, 4, cudaMemcpyDeviceToHost, s));
  GS_CK(cudaStreamSynchronize(s));
  if (!flags) return GSC_OK;
  GS_CK(cudaMemsetAsync(err, 0, 4, s));
  GS_CK(cudaStreamSynchronize(s));
  if (flags & GS_DEVERR_TIMEOUT) {
    set_error("gsc_sort_pairs_u64_static: a bounded look-back wait gave up; the output is not sorted");
    return GSC_ERR_TIMEOUT;
  }
  set_error("gsc_sort_pairs_u64_static: a device-side bounds check failed; the output is not sorted");
  return GSC_ERR_CUDA;
}

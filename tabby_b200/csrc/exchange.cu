// Peer-memory exchange for the vocab-sharded merge (declared in include/tabby_sample.h).
//
// Each rank allocates one exchange buffer and shares it with the other ranks of the job
// through a CUDA IPC handle (the caller moves the 64-byte handles between processes, e.g.
// with torch.distributed.all_gather_object). After tabby_exchange_open every rank holds
// device pointers to every rank's buffer, and tabby_exchange_merge_async runs the merge
// with the exchange inside the kernel: one release/acquire handshake on flag words, then
// peer loads of the blocks over NVLink (xmerge_kernel). No collective library is involved
// and nothing uses multicast.
//
// Buffer layout (each section 256-byte aligned): two block buffers [max_rows][kBlockLd]
// f32 (step e writes and reads the one of parity e & 1), arrive words [world] u32.
#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include "sampler_internal.h"
#include "tabby_sample.h"

using tabby::DeviceScope;

namespace {

constexpr int kBlockLd = 2 + 2 * TABBY_SHARD_TOP_K;
constexpr int kMaxWorld = TABBY_EXCHANGE_MAX_WORLD;
constexpr uint64_t kTimeoutNs = 500ull * 1000ull * 1000ull;  // bounded waits: 0.5 s

size_t section(size_t b) { return (b + 255) / 256 * 256; }

struct Layout {
  size_t blocks, block_bytes, flags, bytes;
  explicit Layout(int max_rows, int world) {
    blocks = 0;
    block_bytes = section((size_t)max_rows * kBlockLd * 4);
    flags = blocks + 2 * block_bytes;
    bytes = flags + section((size_t)world * 4);
  }
};

thread_local char g_xerror[512] = "";

int xfail(int status, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_xerror, sizeof(g_xerror), fmt, ap);
  va_end(ap);
  return tabby::set_error(status, g_xerror);
}

int xcuda(cudaError_t err, const char *what) {
  return xfail(TABBY_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(err), cudaGetErrorString(err));
}


}  // namespace

struct tabby_exchange {
  int32_t device = 0;
  int32_t world = 1;
  int32_t rank = 0;
  int32_t max_rows = 0;
  Layout lay{0, 1};
  unsigned char *base = nullptr;             // this rank's buffer
  unsigned char *peer_base[kMaxWorld] = {};  // every rank's buffer (this rank's included)
  bool peer_opened[kMaxWorld] = {};          // opened through IPC (to be closed)
  bool open = false;
  uint32_t epoch = 0;
};

extern "C" {

int tabby_exchange_create(int32_t device, int32_t world, int32_t rank, int32_t max_rows,
                          tabby_exchange **out) {
  if (!out) return xfail(TABBY_EINVAL, "out is NULL");
  *out = nullptr;
  if (world < 1 || world > kMaxWorld)
    return xfail(TABBY_EINVAL, "world must be in [1, %d], got %d", kMaxWorld, world);
  if (rank < 0 || rank >= world) return xfail(TABBY_EINVAL, "rank %d outside world %d", rank, world);
  if (max_rows < 1) return xfail(TABBY_EINVAL, "max_rows must be >= 1");
  DeviceScope scope(device);
  if (scope.err != cudaSuccess) return xcuda(scope.err, "cudaSetDevice");
  tabby_exchange *x = new tabby_exchange;
  x->device = device;
  x->world = world;
  x->rank = rank;
  x->max_rows = max_rows;
  x->lay = Layout(max_rows, world);
  cudaError_t err = cudaMalloc((void **)&x->base, x->lay.bytes);
  if (err == cudaSuccess) err = cudaMemset(x->base, 0, x->lay.bytes);
  if (err == cudaSuccess) err = cudaDeviceSynchronize();
  if (err != cudaSuccess) {
    if (x->base) cudaFree(x->base);
    delete x;
    return xcuda(err, "exchange allocation");
  }
  *out = x;
  return TABBY_OK;
}

int tabby_exchange_ipc_handle(tabby_exchange *x, void *handle) {
  if (!x || !handle) return xfail(TABBY_EINVAL, "exchange and handle must not be NULL");
  DeviceScope scope(x->device);
  if (scope.err != cudaSuccess) return xcuda(scope.err, "cudaSetDevice");
  cudaIpcMemHandle_t h;
  cudaError_t err = cudaIpcGetMemHandle(&h, x->base);
  if (err != cudaSuccess) return xcuda(err, "cudaIpcGetMemHandle");
  static_assert(sizeof(h) == TABBY_EXCHANGE_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return TABBY_OK;
}

int tabby_exchange_open(tabby_exchange *x, const void *handles) {
  if (!x || !handles) return xfail(TABBY_EINVAL, "exchange and handles must not be NULL");
  if (x->open) return xfail(TABBY_EINVAL, "exchange is already open");
  DeviceScope scope(x->device);
  if (scope.err != cudaSuccess) return xcuda(scope.err, "cudaSetDevice");
  const unsigned char *hb = static_cast<const unsigned char *>(handles);
  for (int q = 0; q < x->world; q++) {
    if (q == x->rank) {
      x->peer_base[q] = x->base;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, hb + (size_t)q * TABBY_EXCHANGE_HANDLE_BYTES, sizeof(h));
    void *p = nullptr;
    cudaError_t err = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (err != cudaSuccess) {
      for (int r = 0; r < q; r++)
        if (x->peer_opened[r]) {
          cudaIpcCloseMemHandle(x->peer_base[r]);
          x->peer_opened[r] = false;
        }
      return xcuda(err, "cudaIpcOpenMemHandle");
    }
    x->peer_base[q] = static_cast<unsigned char *>(p);
    x->peer_opened[q] = true;
  }
  x->open = true;
  return TABBY_OK;
}

int tabby_exchange_blocks(tabby_exchange *x, float **d_blocks, int32_t *block_ld) {
  if (!x || !d_blocks || !block_ld) return xfail(TABBY_EINVAL, "arguments must not be NULL");
  // The buffer the next merge reads: the parity of the next epoch.
  const uint32_t next = x->epoch + 1u;
  *d_blocks = reinterpret_cast<float *>(x->base + x->lay.blocks + (next & 1u) * x->lay.block_bytes);
  *block_ld = kBlockLd;
  return TABBY_OK;
}

int tabby_exchange_merge_async(tabby_exchange *x, int32_t rows,
                               const tabby_sampling_params *d_params, const double *d_uniforms,
                               tabby_sample_outcome *d_out, void *stream) {
  if (!x) return xfail(TABBY_EINVAL, "exchange is NULL");
  if (!x->open) return xfail(TABBY_EINVAL, "exchange is not open (tabby_exchange_open)");
  if (rows < 0 || rows > x->max_rows)
    return xfail(TABBY_EINVAL, "rows must be in [0, %d], got %d", x->max_rows, rows);
  if (rows > 0 && (!d_params || !d_uniforms || !d_out))
    return xfail(TABBY_EINVAL, "params, uniforms and out must not be NULL");
  DeviceScope scope(x->device);
  if (scope.err != cudaSuccess) return xcuda(scope.err, "cudaSetDevice");
  // Every rank makes the same calls in the same order, so the epochs agree. The flag words
  // start at 0 and the first epoch is 1; after a wrap to 0 they hold 0xffffffff, so no
  // word ever matches an epoch its rank has not announced.
  ++x->epoch;
  tabby::XMergeLaunch l;
  l.m.rows = rows;
  l.m.shards = x->world;
  l.m.block_ld = kBlockLd;
  l.m.params = d_params;
  l.m.uniforms = d_uniforms;
  l.m.out = d_out;
  const size_t par = (x->epoch & 1u) * x->lay.block_bytes;
  for (int q = 0; q < x->world; q++) {
    l.peer_blocks[q] = reinterpret_cast<const float *>(x->peer_base[q] + x->lay.blocks + par);
    l.peer_flags[q] = reinterpret_cast<uint32_t *>(x->peer_base[q] + x->lay.flags);
  }
  l.flags = reinterpret_cast<uint32_t *>(x->base + x->lay.flags);
  l.rank = x->rank;
  l.world = x->world;
  l.epoch = x->epoch;
  l.timeout_ns = kTimeoutNs;
  cudaError_t err = tabby::launch_xmerge(l, (cudaStream_t)stream);
  if (err != cudaSuccess) {
    // Nothing was announced: keep this rank's epoch where the peers expect it.
    --x->epoch;
    return xcuda(err, "xmerge_kernel launch");
  }
  return TABBY_OK;
}

int tabby_exchange_destroy(tabby_exchange *x) {
  if (!x) return TABBY_OK;
  DeviceScope scope(x->device);
  for (int q = 0; q < x->world; q++)
    if (x->peer_opened[q]) cudaIpcCloseMemHandle(x->peer_base[q]);
  if (x->base) cudaFree(x->base);
  delete x;
  return TABBY_OK;
}

}  // extern "C"

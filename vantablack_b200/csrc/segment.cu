// segment.cu -- batched dispatch on a context: the counterpart of the Metal
// bridge's vtb_metal_segment_* (src/metal/bridge.h:72-183), where the caller
// chains operations into one MTLCommandBuffer and commits once.
//
// Here a segment records its operations on the host (nothing is launched while
// it is open).  vtb_cuda_segment_commit turns the list into one CUDA graph and
// launches it on the context stream without waiting; vtb_cuda_wait_idle is
// the drain, as on Metal.  A decode loop issues the same list every token
// (same buffers, same shapes), so the context keeps the instantiated graphs of
// the last few distinct lists and a repeated list is a single graph launch.
//
// Inside the graph the matmuls keep programmatic dependent launch between
// them.  Read-backs (segment_copy_d2h) into pinned host memory that the device
// can address are gathered into one kernel that stores straight into host
// memory, at the end of the segment (or before a later operation rewrites a
// source): one launch instead of a copy-engine round trip per buffer.  Other
// read-backs hang off the operation before them on a side branch, so the
// copy engine drains them while the next matmuls run; when a later operation
// writes the bytes being read back, the main chain waits for that copy first.
#include <algorithm>
#include <climits>
#include <cstring>
#include <vector>

namespace vtb {

enum SegKind : int { SEG_MATMUL = 1, SEG_COPY = 2, SEG_H2D = 3, SEG_D2H = 4 };

struct SegOp {
  int kind, q;
  const void* src;  // matmul: weights (offset applied); copies: source
  void* dst;        // matmul: out; copies: destination (host for D2H)
  const void* acts;
  size_t m, k, bytes;
  void* dst_dev;    // D2H into device-addressable pinned memory: the device view of dst
};

// Gathered read-back: copy i moves bytes[i] from src[i] (device) to dst[i]
// (device view of pinned host memory); gridDim.y CTAs share a copy, so many
// host-bound stores are in flight at once.
constexpr int kGatherMax = 96;
struct GatherArgs {
  const char* src[kGatherMax];
  char* dst[kGatherMax];
  unsigned bytes[kGatherMax];
};

__global__ void __launch_bounds__(256) seg_gather_kernel(const __grid_constant__ GatherArgs a) {
  const char* s = a.src[blockIdx.x];
  char* d = a.dst[blockIdx.x];
  const unsigned n = a.bytes[blockIdx.x];
  const unsigned t0 = blockIdx.y * blockDim.x + threadIdx.x, nt = gridDim.y * blockDim.x;
  if (((reinterpret_cast<uintptr_t>(s) | reinterpret_cast<uintptr_t>(d)) & 15u) == 0) {
    const unsigned n16 = n / 16;
    for (unsigned i = t0; i < n16; i += nt) reinterpret_cast<int4*>(d)[i] = __ldg(reinterpret_cast<const int4*>(s) + i);
    for (unsigned i = n16 * 16 + t0; i < n; i += nt) d[i] = s[i];
  } else {
    for (unsigned i = t0; i < n; i += nt) d[i] = s[i];
  }
}

static bool same_ops(const std::vector<SegOp>& a, const std::vector<SegOp>& b) {
  return a.size() == b.size() && (a.empty() || std::memcmp(a.data(), b.data(), a.size() * sizeof(SegOp)) == 0);
}

}  // namespace vtb

struct VtbCudaSeg {
  VtbCudaCtx* ctx;
  std::vector<vtb::SegOp> ops;
  int status;  // first enqueue error (reported by commit)
  bool open;
};

struct VtbSegCache {
  VtbCudaSeg seg;
  struct Entry {
    std::vector<vtb::SegOp> key;
    cudaGraphExec_t exec;
    unsigned long long used;
  };
  std::vector<Entry> entries;
  unsigned long long clock = 0;
  cudaStream_t side = nullptr;
  std::vector<cudaEvent_t> events;
};

namespace vtb {

constexpr int kSegCacheEntries = 8;

static void seg_fail(VtbCudaSeg* s, int status, const char* msg) {
  if (s && s->status == VTB_CUDA_OK) s->status = set_err(status, msg);
}

static cudaEvent_t seg_event(VtbSegCache* c, size_t i) {
  while (c->events.size() <= i) {
    cudaEvent_t e = nullptr;
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return nullptr;
    c->events.push_back(e);
  }
  return c->events[i];
}

static bool ranges_overlap(const void* a, size_t na, const void* b, size_t nb) {
  const char *pa = static_cast<const char*>(a), *pb = static_cast<const char*>(b);
  return pa < pb + nb && pb < pa + na;
}

// Issues the segment's operations on the context stream (inside a capture, or
// eagerly when capture is not possible).  Returns the first CUDA error.
static cudaError_t seg_issue(VtbCudaCtx* ctx, VtbSegCache* c, const std::vector<SegOp>& ops, bool fork_d2h) {
  cudaStream_t st = ctx->stream;
  size_t ev = 0;
  bool side_used = false;
  std::vector<size_t> pend;  // gathered read-backs not yet issued
  auto flush = [&]() -> cudaError_t {
    for (size_t b = 0; b < pend.size(); b += kGatherMax) {
      GatherArgs ga;
      std::memset(&ga, 0, sizeof ga);
      const int n = (int)std::min<size_t>(kGatherMax, pend.size() - b);
      for (int j = 0; j < n; ++j) {
        const SegOp& d = ops[pend[b + j]];
        ga.src[j] = static_cast<const char*>(d.src);
        ga.dst[j] = static_cast<char*>(d.dst_dev);
        ga.bytes[j] = (unsigned)d.bytes;
      }
      size_t most = 0;
      for (int j = 0; j < n; ++j) most = std::max<size_t>(most, ga.bytes[j]);
      const unsigned per = (unsigned)std::min<size_t>(16, (most + 4095) / 4096);  // ~4 KB per CTA
      seg_gather_kernel<<<dim3(n, per ? per : 1), 256, 0, st>>>(ga);
      const cudaError_t e = cudaGetLastError();
      if (e != cudaSuccess) return e;
    }
    pend.clear();
    return cudaSuccess;
  };
  for (size_t i = 0; i < ops.size(); ++i) {
    const SegOp& o = ops[i];
    cudaError_t e = cudaSuccess;
    if (!pend.empty() && o.kind != SEG_D2H) {  // keep a gathered read-back ahead of a write to its source
      const size_t nb = o.kind == SEG_MATMUL ? o.m * 4 : o.bytes;
      for (size_t j : pend)
        if (ranges_overlap(o.dst, nb, ops[j].src, ops[j].bytes)) {
          e = flush();
          break;
        }
      if (e != cudaSuccess) return e;
    }
    switch (o.kind) {
      case SEG_MATMUL:
        e = o.q == Q4_K ? launch_gemv_q4k_mma(o.src, (const float*)o.acts, (float*)o.dst, (int)o.m, (int)o.k, st, true, 0,
                                              nullptr, 0.f, nullptr)
                        : launch_gemv(o.q, o.src, (const float*)o.acts, (float*)o.dst, (int)o.m, (int)o.k, st, true, 0);
        break;
      case SEG_COPY:
        e = cudaMemcpyAsync(o.dst, o.src, o.bytes, cudaMemcpyDeviceToDevice, st);
        break;
      case SEG_H2D:
        e = cudaMemcpyAsync(o.dst, o.src, o.bytes, cudaMemcpyHostToDevice, st);
        break;
      case SEG_D2H: {
        if (!fork_d2h) {
          e = cudaMemcpyAsync(o.dst, o.src, o.bytes, cudaMemcpyDeviceToHost, st);
          break;
        }
        if (o.dst_dev && o.bytes <= 0xffffffffu) {
          pend.push_back(i);
          break;
        }
        // side branch after everything issued so far
        cudaEvent_t a = seg_event(c, ev++), b = seg_event(c, ev++);
        if (!a || !b) return cudaErrorMemoryAllocation;
        e = cudaEventRecord(a, st);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(c->side, a, 0);
        if (e == cudaSuccess) e = cudaMemcpyAsync(o.dst, o.src, o.bytes, cudaMemcpyDeviceToHost, c->side);
        side_used = true;
        bool rewritten = false;  // does a later operation write what this copy reads?
        for (size_t j = i + 1; j < ops.size() && !rewritten; ++j) {
          const SegOp& p = ops[j];
          const size_t nb = p.kind == SEG_MATMUL ? p.m * 4 : p.bytes;
          if (p.kind != SEG_D2H && ranges_overlap(p.dst, nb, o.src, o.bytes)) rewritten = true;
        }
        if (e == cudaSuccess && rewritten) {
          e = cudaEventRecord(b, c->side);
          if (e == cudaSuccess) e = cudaStreamWaitEvent(st, b, 0);
        }
        break;
      }
      default:
        e = cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
  }
  if (cudaError_t e = flush(); e != cudaSuccess) return e;
  if (side_used) {  // join the read-back branch
    cudaEvent_t j = seg_event(c, ev++);
    if (!j) return cudaErrorMemoryAllocation;
    cudaError_t e = cudaEventRecord(j, c->side);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(st, j, 0);
    return e;
  }
  return cudaSuccess;
}

static VtbSegCache* seg_cache(VtbCudaCtx* c) {
  if (!c->seg) {
    VtbSegCache* s = new (std::nothrow) VtbSegCache();
    if (!s) return nullptr;
    if (cudaStreamCreateWithFlags(&s->side, cudaStreamNonBlocking) != cudaSuccess) {
      delete s;
      return nullptr;
    }
    s->seg.ctx = c;
    s->seg.status = VTB_CUDA_OK;
    s->seg.open = false;
    c->seg = s;
  }
  return c->seg;
}

void seg_cache_destroy(VtbSegCache* s) {
  if (!s) return;
  for (auto& e : s->entries) cudaGraphExecDestroy(e.exec);
  for (cudaEvent_t e : s->events) cudaEventDestroy(e);
  if (s->side) cudaStreamDestroy(s->side);
  delete s;
}

static VtbCudaSeg* seg_open(VtbCudaSeg* s) { return s && s->open ? s : nullptr; }

static void seg_matmul(int q, VtbCudaSeg* s, VtbCudaBuf* out, VtbCudaBuf* w, size_t w_off, VtbCudaBuf* acts, size_t m,
                       size_t k) {
  if (!seg_open(s)) return;
  if (!out || !w || !acts) return seg_fail(s, VTB_CUDA_ERR_INVALID_ARG, "segment matmul: null buffer");
  const int64_t rb = host_row_bytes(q, (int64_t)k);
  if (rb <= 0 || m == 0 || m > (size_t)INT_MAX || k > (size_t)INT_MAX || k % host_block_elems(q) ||
      w_off + (size_t)rb * m > w->size || out->size < m * 4 || acts->size < k * 4)
    return seg_fail(s, VTB_CUDA_ERR_INVALID_ARG, "segment matmul: buffer too small for m x k");
  const char* wp = static_cast<const char*>(w->ptr) + w_off;
  if ((reinterpret_cast<uintptr_t>(wp) & 15u) || (reinterpret_cast<uintptr_t>(acts->ptr) & 15u))
    return seg_fail(s, VTB_CUDA_ERR_INVALID_ARG, "segment matmul: weights / activations not 16-byte aligned");
  SegOp o;
  std::memset(&o, 0, sizeof o);  // the list is compared bytewise
  o.kind = SEG_MATMUL;
  o.q = q;
  o.src = wp;
  o.dst = out->ptr;
  o.acts = acts->ptr;
  o.m = m;
  o.k = k;
  s->ops.push_back(o);
}

static void seg_copy(VtbCudaSeg* s, int kind, void* dst, const void* src, size_t bytes) {
  if (!seg_open(s)) return;
  SegOp o;
  std::memset(&o, 0, sizeof o);
  o.kind = kind;
  o.dst = dst;
  o.src = src;
  o.bytes = bytes;
  s->ops.push_back(o);
}

}  // namespace vtb

extern "C" {

VtbCudaSeg* vtb_cuda_segment_begin(VtbCudaCtx* ctx) {
  if (!use_ctx(ctx)) {
    set_err(VTB_CUDA_ERR_INVALID_ARG, "null context");
    return nullptr;
  }
  VtbSegCache* c = vtb::seg_cache(ctx);
  if (!c) {
    set_err(VTB_CUDA_ERR_OOM, "cannot create the segment state");
    return nullptr;
  }
  c->seg.ops.clear();
  c->seg.status = VTB_CUDA_OK;
  c->seg.open = true;
  return &c->seg;
}

void vtb_cuda_segment_matmul_q8_0(VtbCudaSeg* s, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m,
                                  size_t k) {
  vtb::seg_matmul(vtb::Q8_0, s, o, w, off, a, m, k);
}
void vtb_cuda_segment_matmul_q4_k(VtbCudaSeg* s, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m,
                                  size_t k) {
  vtb::seg_matmul(vtb::Q4_K, s, o, w, off, a, m, k);
}
void vtb_cuda_segment_matmul_q5_k(VtbCudaSeg* s, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m,
                                  size_t k) {
  vtb::seg_matmul(vtb::Q5_K, s, o, w, off, a, m, k);
}
void vtb_cuda_segment_matmul_q6_k(VtbCudaSeg* s, VtbCudaBuf* o, VtbCudaBuf* w, size_t off, VtbCudaBuf* a, size_t m,
                                  size_t k) {
  vtb::seg_matmul(vtb::Q6_K, s, o, w, off, a, m, k);
}

void vtb_cuda_segment_copy(VtbCudaSeg* s, VtbCudaBuf* dst, size_t dst_off, VtbCudaBuf* src, size_t src_off,
                           size_t n_floats) {
  if (!vtb::seg_open(s)) return;
  const size_t bytes = n_floats * 4;
  if (!dst || !src || (dst_off | src_off) & 3u || dst_off + bytes > dst->size || src_off + bytes > src->size)
    return vtb::seg_fail(s, VTB_CUDA_ERR_INVALID_ARG, "segment copy: bad range");
  vtb::seg_copy(s, vtb::SEG_COPY, static_cast<char*>(dst->ptr) + dst_off, static_cast<const char*>(src->ptr) + src_off,
                bytes);
}

void vtb_cuda_segment_copy_h2d(VtbCudaSeg* s, VtbCudaBuf* dst, size_t dst_off, const void* host_src, size_t bytes) {
  if (!vtb::seg_open(s)) return;
  if (!dst || !host_src || dst_off + bytes > dst->size)
    return vtb::seg_fail(s, VTB_CUDA_ERR_INVALID_ARG, "segment h2d copy: bad range");
  vtb::seg_copy(s, vtb::SEG_H2D, static_cast<char*>(dst->ptr) + dst_off, host_src, bytes);
}

void vtb_cuda_segment_copy_d2h(VtbCudaSeg* s, void* host_dst, VtbCudaBuf* src, size_t src_off, size_t bytes) {
  if (!vtb::seg_open(s)) return;
  if (!src || !host_dst || src_off + bytes > src->size)
    return vtb::seg_fail(s, VTB_CUDA_ERR_INVALID_ARG, "segment d2h copy: bad range");
  vtb::seg_copy(s, vtb::SEG_D2H, host_dst, static_cast<const char*>(src->ptr) + src_off, bytes);
  // pinned host memory the device can address (cudaHostAlloc'd / registered as mapped)
  cudaPointerAttributes pa;
  if (cudaPointerGetAttributes(&pa, host_dst) == cudaSuccess && pa.type == cudaMemoryTypeHost && pa.devicePointer)
    s->ops.back().dst_dev = pa.devicePointer;
  cudaGetLastError();
}

int vtb_cuda_segment_commit(VtbCudaSeg* s) {
  if (!vtb::seg_open(s)) return set_err(VTB_CUDA_ERR_INVALID_ARG, "no open segment");
  s->open = false;
  if (s->status != VTB_CUDA_OK) return s->status;
  VtbCudaCtx* ctx = s->ctx;
  if (!use_ctx(ctx)) return set_err(VTB_CUDA_ERR_DEVICE, "cannot bind the context's device");
  cudaGetLastError();
  VtbSegCache* c = ctx->seg;
  if (s->ops.empty()) return VTB_CUDA_OK;
  ++c->clock;
  for (auto& e : c->entries)
    if (vtb::same_ops(e.key, s->ops)) {
      e.used = c->clock;
      return cuda_status(cudaGraphLaunch(e.exec, ctx->stream));
    }
  // New list: capture it into a graph.
  cudaGraph_t g = nullptr;
  cudaGraphExec_t ex = nullptr;
  cudaError_t e = cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal);
  if (e == cudaSuccess) {
    const cudaError_t ei = vtb::seg_issue(ctx, c, s->ops, true);
    e = cudaStreamEndCapture(ctx->stream, &g);
    if (ei != cudaSuccess) e = ei;
  }
  if (e == cudaSuccess) e = cudaGraphInstantiate(&ex, g, 0);
  if (g) cudaGraphDestroy(g);
  if (e != cudaSuccess) {  // e.g. a pageable host buffer in a copy: run the list eagerly instead
    cudaGetLastError();
    if (ex) cudaGraphExecDestroy(ex);
    return cuda_status(vtb::seg_issue(ctx, c, s->ops, false));
  }
  if ((int)c->entries.size() >= vtb::kSegCacheEntries) {  // evict the least recently used list
    size_t lru = 0;
    for (size_t i = 1; i < c->entries.size(); ++i)
      if (c->entries[i].used < c->entries[lru].used) lru = i;
    cudaGraphExecDestroy(c->entries[lru].exec);
    c->entries.erase(c->entries.begin() + lru);
  }
  c->entries.push_back({s->ops, ex, c->clock});
  return cuda_status(cudaGraphLaunch(ex, ctx->stream));
}

}  // extern "C"

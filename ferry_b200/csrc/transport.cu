// transport.cu -- kernel 4: expert-parallel dispatch and combine.
//
// Reference-compatible ops (ferry/csrc/expert_ops.cpp):
//   pack_dispatch    :50-66  packet = [hidden bf16 | k weights bf16 | k ids u8]
//   unpack_dispatch  :68-73
//   reduce_partials  :76-83  float32 sum per receive row, in part order, -> bf16
//   scatter_returned :86-92  float32 sum per token, in packet order, -> bf16
//
// Fused path (replaces Transport.dispatch/combine, ferry/transport.py:22-38,
// and its two NCCL all_to_all_single calls): every rank writes its packets
// straight into the owner's receive buffers with 16-byte stores (P2P over
// NVSwitch when the owner is another GPU), raises a sequence-number flag per
// (owner, source), and the owner gathers the routed rows into expert order.
// After the expert GEMM, the owner sums each packet's routes (ascending expert
// order, float32 -> bf16, as reduce_partials) and stores the partial into the
// source's return buffer; the source sums the partials of its peers in rank
// order (float32 -> bf16, as scatter_returned).  Buffers are double-buffered
// by layer parity.  Every wait on a flag is bounded and reports
// DEV_WAIT_TIMEOUT instead of hanging.
#include "common.cuh"
#include "transport.cuh"

namespace ferryb {

__device__ __forceinline__ bool wait_flags(const uint64_t* flags, int n, uint64_t seq, int* err,
                                           uint64_t limit_ns) {
  return wait_flags_bounded(flags, n, seq, err, limit_ns ? limit_ns : 2000000000ull);
}

// True when this rank's expert GEMM or transport recorded an error for the
// data the combine is about to sum.
__device__ __forceinline__ bool poisoned(const FusedArgs& a) {
  if (!a.poison) return false;
  const volatile int* w = a.poison;
  return (w[0] | w[1]) != 0;
}

__device__ __forceinline__ uint4 nan_bf16x8() {
  const uint32_t q = 0x7FC07FC0u;  // two bf16 quiet NaNs
  return make_uint4(q, q, q, q);
}

// ---------------------------------------------------------------------------
// Compat: pack_dispatch / unpack_dispatch.  One CTA per packet.  A packet is
// [hidden bf16 x H | weights bf16 x K | ids u8 x K] with no padding
// (2H + 3K bytes, ferry/csrc/expert_ops.cpp:50-73), so packet rows are only
// as aligned as that stride: the hidden bytes move in pieces of V bytes, V the
// largest power of two <= 8 dividing the stride and the packet base (chosen
// on the host), and the bf16 weights move bytewise.
template <class V>
__device__ __forceinline__ void copy_pieces(uint8_t* dst, const uint8_t* src, int64_t bytes) {
  for (int64_t v = threadIdx.x; v < bytes / (int64_t)sizeof(V); v += blockDim.x)
    reinterpret_cast<V*>(dst)[v] = reinterpret_cast<const V*>(src)[v];
}

template <class V>
__global__ void pack_dispatch_kernel(const __nv_bfloat16* __restrict__ hidden, int64_t tokens,
                                     int64_t H, const int64_t* __restrict__ selected,
                                     const __nv_bfloat16* __restrict__ weights, int64_t K_sel,
                                     const int64_t* __restrict__ send_idx,
                                     const int64_t* __restrict__ send_ids, int64_t K,
                                     int64_t experts, uint8_t* __restrict__ payload, int* err) {
  const int64_t i = blockIdx.x;
  const int64_t t = send_idx[i];
  const int64_t stride = 2 * H + 3 * K;
  uint8_t* row = payload + i * stride;
  if (t < 0 || t >= tokens) {
    if (threadIdx.x == 0) atomicCAS(err, 0, DEV_BAD_INPUT);
    return;
  }
  copy_pieces<V>(row, reinterpret_cast<const uint8_t*>(hidden + t * H), 2 * H);
  if (threadIdx.x < K) {
    const int j = threadIdx.x;
    const int64_t e = send_ids[i * K + j];
    __nv_bfloat16 w = __float2bfloat16_rn(0.0f);
    if (e >= 0) {
      if (e >= experts) atomicCAS(err, 0, DEV_BAD_INPUT);
      // dense[t, e] = bf16(float32 sum of the token's weights for e)
      float acc = 0.0f;
      for (int64_t jj = 0; jj < K_sel; ++jj)
        if (selected[t * K_sel + jj] == e) acc += __bfloat162float(weights[t * K_sel + jj]);
      w = __float2bfloat16_rn(acc);
    }
    const uint16_t bits = __bfloat16_as_ushort(w);
    row[2 * H + 2 * j] = static_cast<uint8_t>(bits & 0xff);
    row[2 * H + 2 * j + 1] = static_cast<uint8_t>(bits >> 8);
    row[2 * H + 2 * K + j] = static_cast<uint8_t>(e);
  }
}

template <class V>
__global__ void unpack_dispatch_kernel(const uint8_t* __restrict__ raw, int64_t m, int64_t H,
                                       int64_t K, __nv_bfloat16* __restrict__ x,
                                       __nv_bfloat16* __restrict__ w) {
  const int64_t i = blockIdx.x;
  const uint8_t* row = raw + i * (2 * H + 3 * K);
  copy_pieces<V>(reinterpret_cast<uint8_t*>(x + i * H), row, 2 * H);
  if (threadIdx.x < K) {
    const int j = threadIdx.x;
    const uint16_t bits = static_cast<uint16_t>(row[2 * H + 2 * j]) |
                          static_cast<uint16_t>(row[2 * H + 2 * j + 1]) << 8;
    w[i * K + j] = __ushort_as_bfloat16(bits);
  }
}

// largest power of two <= 8 dividing the packet stride and both bases (hidden
// rows are 2H bytes apart, a multiple of 8)
static int packet_align(int64_t stride, const void* packets, const void* rows) {
  const uint64_t v = static_cast<uint64_t>(stride) | reinterpret_cast<uintptr_t>(packets) |
                     reinterpret_cast<uintptr_t>(rows) | 8u;
  return static_cast<int>(v & (~v + 1));
}

// ---------------------------------------------------------------------------
// Ordered segment sums used by reduce_partials and scatter_returned:
// dst[k] = bf16(sum over p ascending with keys[p] == k of float(src[p])).
__global__ void seg_count_kernel(const int64_t* keys, int64_t n, int64_t n_keys, int* cnt,
                                 int* err) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < n;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[p];
    if (k < 0 || k >= n_keys) { atomicCAS(err, 0, DEV_BAD_INPUT); continue; }
    atomicAdd(&cnt[k], 1);
  }
}

// single-CTA exclusive scan over n_keys counters (chunks of 1024)
__global__ void seg_scan_kernel(const int* cnt, int64_t n_keys, int* off) {
  __shared__ int warp_sum[32];
  __shared__ int carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int64_t base = 0; base < n_keys; base += blockDim.x) {
    const int64_t k = base + threadIdx.x;
    const int v = k < n_keys ? cnt[k] : 0;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sum[warp] = x;
    __syncthreads();
    if (warp == 0) {
      const int w = lane < (int)(blockDim.x >> 5) ? warp_sum[lane] : 0;
      int wx = w;
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, wx, o);
        if (lane >= o) wx += y;
      }
      warp_sum[lane] = wx - w;
    }
    __syncthreads();
    if (k < n_keys) off[k] = carry + warp_sum[warp] + x - v;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry += warp_sum[warp] + x;
    __syncthreads();
  }
  if (threadIdx.x == 0) off[n_keys] = carry;
}

__global__ void seg_fill_kernel(const int64_t* keys, int64_t n, int64_t n_keys, const int* off,
                                int* cursor, int* order) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < n;
       p += (int64_t)gridDim.x * blockDim.x) {
    const int64_t k = keys[p];
    if (k < 0 || k >= n_keys) continue;
    order[off[k] + atomicAdd(&cursor[k], 1)] = (int)p;
  }
}

// One CTA per key: sort the key's positions ascending, then sum in that order.
__global__ void seg_sum_kernel(const __nv_bfloat16* __restrict__ src, int64_t H, const int* off,
                               int* order, __nv_bfloat16* __restrict__ dst) {
  const int64_t k = blockIdx.x;
  const int a = off[k], b = off[k + 1];
  if (threadIdx.x == 0) {
    for (int i = a + 1; i < b; ++i) {
      const int v = order[i];
      int j = i;
      while (j > a && order[j - 1] > v) { order[j] = order[j - 1]; --j; }
      order[j] = v;
    }
  }
  __syncthreads();
  for (int64_t c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
    for (int i = a; i < b; ++i) {
      const uint4 v = *reinterpret_cast<const uint4*>(src + (int64_t)order[i] * H + c);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(e[q]);
    }
    uint4 o;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16_rn(acc[q]);
    *reinterpret_cast<uint4*>(dst + k * H + c) = o;
  }
}

static int64_t a256(int64_t b) { return (b + 255) & ~int64_t(255); }

SymLayout sym_layout(int world, int T, int K, int H, int E) {
  SymLayout l{};
  size_t o = 0;
  const size_t rows = (size_t)world * T;
  l.recv_x = o; o += a256(rows * H * 2);
  l.recv_w = o; o += a256(rows * K * 2);
  l.recv_ids = o; o += a256(rows * K);
  l.ret = o; o += a256(rows * H * 2);
  l.dflag = o; o += a256(world * 8);
  l.cflag = o; o += a256(world * 8);
  l.gather_ids = o; o += a256(rows * K);
  l.gather_hist = o; o += a256((size_t)world * E * 4);
  l.gflag = o; o += a256(world * 8);
  l.half = o;
  return l;
}

int64_t seg_workspace(int64_t n, int64_t n_keys) {
  return a256((n_keys + 1) * 4) * 2 + a256(n_keys * 4) + a256(n * 4) + 256;
}

int ordered_segment_sum(const __nv_bfloat16* src, const int64_t* keys, int64_t n, int64_t n_keys,
                        int64_t H, __nv_bfloat16* dst, void* ws, int64_t ws_bytes,
                        cudaStream_t stream) {
  FB_CHECK_ARG(H % 8 == 0, "hidden must be a multiple of 8");
  FB_CHECK_ARG(ws && ws_bytes >= seg_workspace(n, n_keys), "segment-sum workspace too small");
  if (n_keys == 0) return FERRYB_OK;
  uint8_t* b = static_cast<uint8_t*>(ws);
  int* cnt = reinterpret_cast<int*>(b);
  int* off = reinterpret_cast<int*>(b + a256((n_keys + 1) * 4));
  int* cursor = reinterpret_cast<int*>(b + 2 * a256((n_keys + 1) * 4));
  int* order = reinterpret_cast<int*>(b + 2 * a256((n_keys + 1) * 4) + a256(n_keys * 4));
  int* err = reinterpret_cast<int*>(b + 2 * a256((n_keys + 1) * 4) + a256(n_keys * 4) + a256(n * 4));
  FB_CUDA(cudaMemsetAsync(cnt, 0, n_keys * 4, stream));
  FB_CUDA(cudaMemsetAsync(cursor, 0, n_keys * 4, stream));
  FB_CUDA(cudaMemsetAsync(err, 0, 4, stream));
  const int blocks = (int)std::min<int64_t>(1024, (n + 255) / 256 + 1);
  if (n > 0) seg_count_kernel<<<blocks, 256, 0, stream>>>(keys, n, n_keys, cnt, err);
  seg_scan_kernel<<<1, 1024, 0, stream>>>(cnt, n_keys, off);
  if (n > 0) seg_fill_kernel<<<blocks, 256, 0, stream>>>(keys, n, n_keys, off, cursor, order);
  seg_sum_kernel<<<(unsigned)n_keys, 256, 0, stream>>>(src, H, off, order, dst);
  FB_LAUNCH_CHECK();
  int h_err = 0;
  FB_CUDA(cudaMemcpyAsync(&h_err, err, 4, cudaMemcpyDeviceToHost, stream));
  FB_CUDA(cudaStreamSynchronize(stream));
  if (h_err) return fail(FERRYB_EINVAL, "index out of range in reduce/scatter");
  return FERRYB_OK;
}

// ---------------------------------------------------------------------------
// Fused path.
// dispatch: one CTA per local token; for each peer with a packet, write the
// token's hidden row, the weights of its routes to that peer (ascending id
// order) and the ids into the peer's receive buffers at the packet's row.
__global__ void fused_dispatch_kernel(const FusedArgs a) {
  const int t = blockIdx.x;
  const int R = a.world, K = a.topk, H = a.hdim;
  const int g = a.rank * a.tokens_per_rank + t;
  __shared__ int ids_s[kMaxTopK], pos_s[kMaxTopK];
  span_begin(a.ts_dispatch);
  for (int p = 0; p < R; ++p) {
    const int row = a.peer_row[t * R + p];
    if (row < 0) continue;
    uint8_t* base = reinterpret_cast<uint8_t*>(a.peer_base[p]) + a.parity * a.buf_stride;
    __nv_bfloat16* rx = reinterpret_cast<__nv_bfloat16*>(base + a.off_recv_x) + (size_t)row * H;
    const uint4* src = reinterpret_cast<const uint4*>(a.hidden + (size_t)t * H);
    for (int v = threadIdx.x; v < H / 8; v += blockDim.x) reinterpret_cast<uint4*>(rx)[v] = src[v];
    if (threadIdx.x == 0) {
      // ids of this packet ascending (ferry/layout.py:27-33) and their token column
      int size = 0;
      for (int j = 0; j < K; ++j) {
        if (a.dest[g * K + j] != p) continue;
        const int e = a.ids[g * K + j];
        int q = size;
        while (q > 0 && ids_s[q - 1] > e) { ids_s[q] = ids_s[q - 1]; pos_s[q] = pos_s[q - 1]; --q; }
        ids_s[q] = e;
        pos_s[q] = j;
        ++size;
      }
      __nv_bfloat16* rw = reinterpret_cast<__nv_bfloat16*>(base + a.off_recv_w) + (size_t)row * K;
      uint8_t* ri = base + a.off_recv_ids + (size_t)row * K;
      for (int j = 0; j < K; ++j) {
        rw[j] = j < size ? a.weights[(size_t)t * K + pos_s[j]] : __float2bfloat16_rn(0.0f);
        ri[j] = j < size ? (uint8_t)ids_s[j] : (uint8_t)0xff;
      }
    }
    __syncthreads();
  }
  span_end(a.ts_dispatch);
}

// Raise this rank's flag in every peer's `flag_off` array (after the
// preceding kernel's stores, which the kernel boundary makes visible).
__global__ void signal_kernel(const FusedArgs a, size_t flag_off, uint64_t seq) {
  const int p = threadIdx.x;
  if (p >= a.world) return;
  __threadfence_system();
  uint64_t* f = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(a.peer_base[p]) +
                                            a.parity * a.buf_stride + flag_off) + a.rank;
  st_release_sys(f, seq);
}

// permute: X[p] = recv_x[rows[p]], W[p] = recv_w[rows[p], cols[p]] (after all
// sources have signalled).  One CTA per 4 routes.
__global__ void fused_permute_kernel(const FusedArgs a, uint64_t seq) {
  uint8_t* base = reinterpret_cast<uint8_t*>(a.local_base) + a.parity * a.buf_stride;
  __shared__ int ok;
  span_begin(a.ts_permute);
  if (threadIdx.x == 0)
    ok = a.world == 1 || wait_flags(reinterpret_cast<const uint64_t*>(base + a.off_dflag), a.world,
                                    seq, a.err, a.wait_ns);
  __syncthreads();
  if (!ok) return;
  const int H = a.hdim, K = a.topk;
  const int n_routes = *a.n_routes_dev;
  const __nv_bfloat16* rx = reinterpret_cast<const __nv_bfloat16*>(base + a.off_recv_x);
  const __nv_bfloat16* rw = reinterpret_cast<const __nv_bfloat16*>(base + a.off_recv_w);
  const int vec = H / 8;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n_routes * vec; i += gridDim.x * blockDim.x) {
    const int p = i / vec, v = i % vec;
    const int64_t row = a.rows[p];
    reinterpret_cast<uint4*>(a.x_sorted + (size_t)p * H)[v] =
        reinterpret_cast<const uint4*>(rx + (size_t)row * H)[v];
    if (v == 0) a.route_w[p] = rw[(size_t)row * K + a.cols[p]];
  }
  __syncthreads();
  span_end(a.ts_permute);
}

// o = bf16(float(o) + float(b)) lane-wise (a torch bf16 add)
__device__ __forceinline__ void add_bf16x8(uint4& o, const uint4 b) {
  __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
  const __nv_bfloat16* be = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
  for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16_rn(__bfloat162float(oe[q]) + __bfloat162float(be[q]));
}

// combine (owner side): per receive row, bf16(sum over its routes in ascending
// expert order of float(out[route])), stored to the source rank's return
// buffer -- or, with one rank, straight into the layer output.
__global__ void fused_combine_kernel(const FusedArgs a) {
  const int row = blockIdx.x;
  const int n_recv = *a.n_recv_dev;
  if (row >= n_recv) return;
  span_begin(a.ts_combine);
  const int H = a.hdim, K = a.topk;
  const int g = a.recv_token[row];
  const int src = g / a.tokens_per_rank, t = g % a.tokens_per_rank;
  __nv_bfloat16* dst;
  const __nv_bfloat16* add = nullptr;
  if (a.world == 1) {
    dst = a.out + (size_t)t * H;
    if (a.addend) add = a.addend + (size_t)t * H;
  } else {
    uint8_t* base = reinterpret_cast<uint8_t*>(a.peer_base[src]) + a.parity * a.buf_stride;
    dst = reinterpret_cast<__nv_bfloat16*>(base + a.off_ret) +
          ((size_t)a.rank * a.tokens_per_rank + t) * H;
  }
  if (poisoned(a)) {
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
      *reinterpret_cast<uint4*>(dst + c) = nan_bf16x8();
    __syncthreads();
    span_end(a.ts_combine);
    return;
  }
  int pos[kMaxTopK];
  int np = 0;
  for (int j = 0; j < K; ++j) {
    const int q = a.csr_pos[(size_t)row * K + j];
    if (q < 0) break;
    pos[np++] = q;
  }
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
    for (int j = 0; j < np; ++j) {
      const uint4 v = *reinterpret_cast<const uint4*>(a.expert_out + (size_t)pos[j] * H + c);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(e[q]);
    }
    uint4 o;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16_rn(acc[q]);
    if (add) add_bf16x8(o, *reinterpret_cast<const uint4*>(add + c));
    *reinterpret_cast<uint4*>(dst + c) = o;
  }
  __syncthreads();
  span_end(a.ts_combine);
}

// final scatter (source side, world > 1): out[t] = bf16(sum over peers p in
// rank order with a packet of float(ret[p][t])); tokens without any route get 0.
// When a peer's partials never arrived (the flag wait ran out) or this rank's
// own GEMM/transport failed, the row is NaN.
__global__ void fused_final_kernel(const FusedArgs a, uint64_t seq) {
  const int t = blockIdx.x;
  uint8_t* base = reinterpret_cast<uint8_t*>(a.local_base) + a.parity * a.buf_stride;
  __shared__ int ok;
  span_begin(a.ts_final);
  if (threadIdx.x == 0)
    ok = wait_flags(reinterpret_cast<const uint64_t*>(base + a.off_cflag), a.world, seq, a.err,
                    a.wait_ns) &&
         !poisoned(a);
  __syncthreads();
  const int H = a.hdim, R = a.world;
  if (!ok) {
    for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8)
      *reinterpret_cast<uint4*>(a.out + (size_t)t * H + c) = nan_bf16x8();
    __syncthreads();
    span_end(a.ts_final);
    return;
  }
  const __nv_bfloat16* ret = reinterpret_cast<const __nv_bfloat16*>(base + a.off_ret);
  for (int c = threadIdx.x * 8; c < H; c += blockDim.x * 8) {
    float acc[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) acc[q] = 0.0f;
    for (int p = 0; p < R; ++p) {
      if (a.peer_row[t * R + p] < 0) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(ret + ((size_t)p * a.tokens_per_rank + t) * H + c);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += __bfloat162float(e[q]);
    }
    uint4 o;
    __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) oe[q] = __float2bfloat16_rn(acc[q]);
    if (a.addend) add_bf16x8(o, *reinterpret_cast<const uint4*>(a.addend + (size_t)t * H + c));
    *reinterpret_cast<uint4*>(a.out + (size_t)t * H + c) = o;
  }
  __syncthreads();
  span_end(a.ts_final);
}

int fused_dispatch(const FusedArgs& a, uint64_t seq, cudaStream_t stream) {
  if (a.tokens_per_rank > 0)
    fused_dispatch_kernel<<<a.tokens_per_rank, 256, 0, stream>>>(a);
  if (a.world > 1 && !(a.skip_signals & 1)) signal_kernel<<<1, 32, 0, stream>>>(a, a.off_dflag, seq);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

int fused_permute(const FusedArgs& a, uint64_t seq, int n_routes_hint, cudaStream_t stream) {
  const int vec = a.hdim / 8;
  int blocks = (int)std::min<int64_t>(1184, ((int64_t)std::max(n_routes_hint, 1) * vec + 255) / 256);
  fused_permute_kernel<<<blocks, 256, 0, stream>>>(a, seq);
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

// With one rank every token has all its routes on this rank, so the combine
// writes every output row.
int fused_combine(const FusedArgs& a, uint64_t seq, int n_recv_hint, cudaStream_t stream,
                  cudaEvent_t after_stores) {
  if (n_recv_hint > 0) fused_combine_kernel<<<n_recv_hint, 256, 0, stream>>>(a);
  if (after_stores) FB_CUDA(cudaEventRecord(after_stores, stream));
  if (a.world > 1) {
    if (!(a.skip_signals & 2)) signal_kernel<<<1, 32, 0, stream>>>(a, a.off_cflag, seq);
    if (a.tokens_per_rank > 0) fused_final_kernel<<<a.tokens_per_rank, 256, 0, stream>>>(a, seq);
  }
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

}  // namespace ferryb

using namespace ferryb;

extern "C" int ferryb_pack_dispatch(const void* hidden, int64_t tokens, int64_t hidden_dim,
                                    const int64_t* selected, const void* weights, int64_t topk,
                                    const int64_t* send_idx, const int64_t* send_ids,
                                    int64_t n_packets, int64_t experts, void* payload, int32_t* err,
                                    cudaStream_t stream) {
  FB_CHECK_ARG(hidden_dim % 4 == 0 && topk >= 1 && topk <= 256 && n_packets >= 0,
               "pack_dispatch: bad sizes");
  if (n_packets == 0) return FERRYB_OK;
  FB_CHECK_ARG(hidden && selected && weights && send_idx && send_ids && payload && err,
               "pack_dispatch: null pointer");
  const auto* hid = static_cast<const __nv_bfloat16*>(hidden);
  const auto* wts = static_cast<const __nv_bfloat16*>(weights);
  auto* out = static_cast<uint8_t*>(payload);
  const unsigned grid = (unsigned)n_packets;
  switch (packet_align(2 * hidden_dim + 3 * topk, payload, hidden)) {
    case 8: pack_dispatch_kernel<uint2><<<grid, 256, 0, stream>>>(hid, tokens, hidden_dim, selected, wts, topk, send_idx, send_ids, topk, experts, out, err); break;
    case 4: pack_dispatch_kernel<uint32_t><<<grid, 256, 0, stream>>>(hid, tokens, hidden_dim, selected, wts, topk, send_idx, send_ids, topk, experts, out, err); break;
    case 2: pack_dispatch_kernel<uint16_t><<<grid, 256, 0, stream>>>(hid, tokens, hidden_dim, selected, wts, topk, send_idx, send_ids, topk, experts, out, err); break;
    default: pack_dispatch_kernel<uint8_t><<<grid, 256, 0, stream>>>(hid, tokens, hidden_dim, selected, wts, topk, send_idx, send_ids, topk, experts, out, err); break;
  }
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int ferryb_unpack_dispatch(const void* raw, int64_t m, int64_t hidden_dim, int64_t topk,
                                      void* x, void* w, cudaStream_t stream) {
  FB_CHECK_ARG(hidden_dim % 4 == 0 && topk >= 1 && topk <= 256 && m >= 0, "unpack: bad sizes");
  if (m == 0) return FERRYB_OK;
  const auto* src = static_cast<const uint8_t*>(raw);
  auto* xo = static_cast<__nv_bfloat16*>(x);
  auto* wo = static_cast<__nv_bfloat16*>(w);
  const unsigned grid = (unsigned)m;
  switch (packet_align(2 * hidden_dim + 3 * topk, raw, x)) {
    case 8: unpack_dispatch_kernel<uint2><<<grid, 256, 0, stream>>>(src, m, hidden_dim, topk, xo, wo); break;
    case 4: unpack_dispatch_kernel<uint32_t><<<grid, 256, 0, stream>>>(src, m, hidden_dim, topk, xo, wo); break;
    case 2: unpack_dispatch_kernel<uint16_t><<<grid, 256, 0, stream>>>(src, m, hidden_dim, topk, xo, wo); break;
    default: unpack_dispatch_kernel<uint8_t><<<grid, 256, 0, stream>>>(src, m, hidden_dim, topk, xo, wo); break;
  }
  FB_LAUNCH_CHECK();
  return FERRYB_OK;
}

extern "C" int64_t ferryb_segment_sum_workspace(int64_t n, int64_t n_keys) {
  return seg_workspace(n, n_keys);
}

extern "C" int ferryb_reduce_partials(const void* parts, const int64_t* rows, int64_t total,
                                      int64_t received, int64_t hidden_dim, void* partial,
                                      void* workspace, int64_t workspace_bytes,
                                      cudaStream_t stream) {
  FB_CHECK_ARG(received >= 0 && total >= 0, "reduce_partials: bad sizes");
  return ordered_segment_sum(static_cast<const __nv_bfloat16*>(parts), rows, total, received,
                             hidden_dim, static_cast<__nv_bfloat16*>(partial), workspace,
                             workspace_bytes, stream);
}

extern "C" int ferryb_scatter_returned(const void* returned, const int64_t* send_idx, int64_t n,
                                       int64_t tokens, int64_t hidden_dim, void* out,
                                       void* workspace, int64_t workspace_bytes,
                                       cudaStream_t stream) {
  FB_CHECK_ARG(n >= 0 && tokens >= 0, "scatter_returned: bad sizes");
  return ordered_segment_sum(static_cast<const __nv_bfloat16*>(returned), send_idx, n, tokens,
                             hidden_dim, static_cast<__nv_bfloat16*>(out), workspace,
                             workspace_bytes, stream);
}

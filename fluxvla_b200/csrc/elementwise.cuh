// Memory-bound helper kernels: row norms, image patchify, token embedding
// gather, and the exact-f32 small linears of the action head.
#pragma once

#include "common.cuh"

namespace fvb {

constexpr int NORM_THREADS = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
  return t;
}

// One CTA per row; dim <= 8 * NORM_THREADS * 4 handled with a strided loop.
__global__ void __launch_bounds__(NORM_THREADS)
    norm_kernel(int mode, const float* __restrict__ x, long long ld_in,
                void* __restrict__ out, long long ld_out, int out_f32,
                int dim, const bf16* __restrict__ w,
                const bf16* __restrict__ b, const float* __restrict__ mod,
                float eps) {
  __shared__ float red[32];
  griddep_wait();
  griddep_launch_dependents();
  const int row = blockIdx.x;
  const float* xr = x + (long long)row * ld_in;
  float s = 0.f, ss = 0.f;
  for (int i = threadIdx.x * 4; i < dim; i += NORM_THREADS * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    s += v.x + v.y + v.z + v.w;
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  float mean = 0.f, rstd;
  if (mode == FVB_NORM_LAYER) {
    mean = block_sum(s, red) / dim;
    // two-pass variance for accuracy
    float q = 0.f;
    for (int i = threadIdx.x * 4; i < dim; i += NORM_THREADS * 4) {
      const float4 v = *reinterpret_cast<const float4*>(xr + i);
      q += (v.x - mean) * (v.x - mean) + (v.y - mean) * (v.y - mean) +
           (v.z - mean) * (v.z - mean) + (v.w - mean) * (v.w - mean);
    }
    rstd = rsqrtf(block_sum(q, red) / dim + eps);
  } else {
    rstd = rsqrtf(block_sum(ss, red) / dim + eps);
  }
  for (int i = threadIdx.x * 4; i < dim; i += NORM_THREADS * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + i);
    float y[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = i + e;
      float t = (y[e] - mean) * rstd;
      if (mode == FVB_NORM_GEMMA_RMS) {
        t *= 1.f + __bfloat162float(w[c]);
      } else if (mode == FVB_NORM_ADA_RMS) {
        t = t * (1.f + mod[c]) + mod[dim + c];
      } else {
        t = t * __bfloat162float(w[c]) + __bfloat162float(b[c]);
      }
      y[e] = t;
    }
    if (out_f32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) +
                                 (long long)row * ld_out + i) =
          make_float4(y[0], y[1], y[2], y[3]);
    } else {
      uint2 pk = make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
      *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(out) +
                                (long long)row * ld_out + i) = pk;
    }
  }
}

// Same norms with one warp per row (8 rows per CTA) for dim % 128 == 0 and
// dim <= 2048: each lane holds its dim/32 values in registers, so the row is
// read once and reduced with shuffles only.
constexpr int NORM_ROWS_PER_CTA = 8;
template <int V4>  // float4 per lane = dim / 128
__global__ void __launch_bounds__(256)
    norm_warp_kernel(int mode, const float* __restrict__ x, long long ld_in,
                     void* __restrict__ out, long long ld_out, int out_f32,
                     int rows, int dim, const bf16* __restrict__ w,
                     const bf16* __restrict__ b, const float* __restrict__ mod,
                     float eps) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * NORM_ROWS_PER_CTA + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float* xr = x + (long long)row * ld_in;
  float4 v[V4];
  float s = 0.f, ss = 0.f;
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    v[i] = *reinterpret_cast<const float4*>(xr + (i * 32 + lane) * 4);
    s += v[i].x + v[i].y + v[i].z + v[i].w;
    ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
  }
  float mean = 0.f, rstd;
  if (mode == FVB_NORM_LAYER) {
    mean = warp_sum(s) / dim;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < V4; ++i)
      q += (v[i].x - mean) * (v[i].x - mean) + (v[i].y - mean) * (v[i].y - mean) +
           (v[i].z - mean) * (v[i].z - mean) + (v[i].w - mean) * (v[i].w - mean);
    rstd = rsqrtf(warp_sum(q) / dim + eps);
  } else {
    rstd = rsqrtf(warp_sum(ss) / dim + eps);
  }
#pragma unroll
  for (int i = 0; i < V4; ++i) {
    const int c0 = (i * 32 + lane) * 4;
    float y[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int c = c0 + e;
      float t = (y[e] - mean) * rstd;
      if (mode == FVB_NORM_GEMMA_RMS) t *= 1.f + __bfloat162float(w[c]);
      else if (mode == FVB_NORM_ADA_RMS) t = t * (1.f + mod[c]) + mod[dim + c];
      else t = t * __bfloat162float(w[c]) + __bfloat162float(b[c]);
      y[e] = t;
    }
    if (out_f32)
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (long long)row * ld_out + c0) =
          make_float4(y[0], y[1], y[2], y[3]);
    else
      *reinterpret_cast<uint2*>(reinterpret_cast<bf16*>(out) + (long long)row * ld_out + c0) =
          make_uint2(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]));
  }
}

// One axis of OpenCV's INTER_LINEAR resize: taps s0, s1 and 11-bit
// fixed-point weights of destination index d (f computed in double without
// contraction, rounded to float, weights rounded half to even).  Along x a
// tap outside [0, src-1) has its fraction forced to 0; along y only the row
// indices are clamped.
__device__ __forceinline__ void resize_taps(int d, int dst, int src, bool clamp_w,
                                            int& s0, int& s1, int& w0, int& w1) {
  const double scale = __drcp_rn(__ddiv_rn((double)dst, (double)src));
  float f = (float)__dadd_rn(__dmul_rn((double)d + 0.5, scale), -0.5);
  int s = (int)floorf(f);
  f -= (float)s;
  if (clamp_w) {
    if (s < 0) { s = 0; f = 0.f; }
    if (s >= src - 1) { s = src - 1; f = 0.f; }
  }
  w0 = (int)rintf(__fmul_rn(1.f - f, 2048.f));
  w1 = (int)rintf(__fmul_rn(f, 2048.f));
  s0 = min(max(s, 0), src - 1);
  s1 = min(max(s + 1, 0), src - 1);
}

// uint8 HWC views of any size -> resized (OpenCV INTER_LINEAR, bit-exact
// uint8) -> normalised -> bf16 patch rows of the size x size image, fused:
// one CTA per patch row, one thread per (channel, ky, kx) element.
__global__ void resize_patchify_kernel(const uint8_t* __restrict__ img, int H,
                                       int W, int size, int P, float m0, float m1,
                                       float m2, float s0, float s1, float s2,
                                       bf16* __restrict__ out, long long ldo) {
  griddep_wait();
  griddep_launch_dependents();
  const int g = size / P;
  const int r = blockIdx.x;
  const int v = r / (g * g), py = (r / g) % g, px = r % g;
  const int K = 3 * P * P;
  const uint8_t* src = img + (long long)v * H * W * 3;
  bf16* o = out + (long long)r * ldo;
  for (int col = threadIdx.x; col < ldo; col += blockDim.x) {
    float val = 0.f;
    if (col < K) {
      const int c = col / (P * P), ky = (col / P) % P, kx = col % P;
      const int y = py * P + ky, x = px * P + kx;
      int x0, x1, a0, a1, y0, y1, b0, b1;
      resize_taps(x, size, W, true, x0, x1, a0, a1);
      resize_taps(y, size, H, false, y0, y1, b0, b1);
      const uint8_t* r0 = src + (long long)y0 * W * 3 + c;
      const uint8_t* r1 = src + (long long)y1 * W * 3 + c;
      const int h0 = r0[x0 * 3] * a0 + r0[x1 * 3] * a1;
      const int h1 = r1[x0 * 3] * a0 + r1[x1 * 3] * a1;
      const int q = (((h0 >> 4) * b0) >> 16) + (((h1 >> 4) * b1) >> 16);
      const int u8 = min(max((q + 2) >> 2, 0), 255);
      const float mean = c == 0 ? m0 : (c == 1 ? m1 : m2);
      const float sd = c == 0 ? s0 : (c == 1 ? s1 : s2);
      val = ((float)u8 - mean) / (sd + 1e-8f);
    }
    o[col] = __float2bfloat16(val);
  }
}

// uint8 HWC images -> normalised bf16 patch rows.  One CTA per patch row.
__global__ void patchify_kernel(const uint8_t* __restrict__ img, int H, int W,
                                int P, float m0, float m1, float m2, float s0,
                                float s1, float s2, bf16* __restrict__ out,
                                long long ldo) {
  griddep_wait();
  griddep_launch_dependents();
  const int gw = W / P, gh = H / P;
  const int r = blockIdx.x;
  const int v = r / (gh * gw), py = (r / gw) % gh, px = r % gw;
  const int K = 3 * P * P;
  bf16* o = out + (long long)r * ldo;
  for (int col = threadIdx.x; col < ldo; col += blockDim.x) {
    float val = 0.f;
    if (col < K) {
      const int c = col / (P * P), ky = (col / P) % P, kx = col % P;
      const int y = py * P + ky, x = px * P + kx;
      const float raw = img[(((long long)v * H + y) * W + x) * 3 + c];
      const float mean = c == 0 ? m0 : (c == 1 ? m1 : m2);
      const float sd = c == 0 ? s0 : (c == 1 ? s1 : s2);
      val = (raw - mean) / (sd + 1e-8f);
    }
    o[col] = __float2bfloat16(val);
  }
}

// Normalised float CHW pixels [views, 3, H, W] (the reference model's
// `images` input after its NormalizeImages transform) -> bf16 patch rows in
// the layout of patchify_kernel.  One CTA per patch row; a warp reads 32
// consecutive x of one (channel, ky) line of the patch.
__global__ void patchify_f32_kernel(const float* __restrict__ pix, int H, int W,
                                    int P, bf16* __restrict__ out,
                                    long long ldo) {
  griddep_wait();
  griddep_launch_dependents();
  const int gw = W / P, gh = H / P;
  const int r = blockIdx.x;
  const int v = r / (gh * gw), py = (r / gw) % gh, px = r % gw;
  const int K = 3 * P * P;
  bf16* o = out + (long long)r * ldo;
  for (int col = threadIdx.x; col < ldo; col += blockDim.x) {
    float val = 0.f;
    if (col < K) {
      const int c = col / (P * P), ky = (col / P) % P, kx = col % P;
      const int y = py * P + ky, x = px * P + kx;
      val = __ldg(pix + (((long long)v * 3 + c) * H + y) * W + x);
    }
    o[col] = __float2bfloat16(val);
  }
}

__global__ void embed_kernel(const long long* __restrict__ ids,
                             const bf16* __restrict__ table, int dim,
                             float scale, float* __restrict__ out,
                             long long ldo) {
  griddep_wait();
  griddep_launch_dependents();
  const long long id = ids[blockIdx.x];
  const bf16* src = table + id * dim;
  float* dst = out + (long long)blockIdx.x * ldo;
  for (int i = threadIdx.x; i < dim; i += blockDim.x)
    dst[i] = __bfloat162float(src[i]) * scale;
}

// One warp per output element (t, n): y = act(x[t,:] . W[n,:] + bias[n]).
__global__ void small_linear_kernel(const float* __restrict__ x, long long ldx,
                                    int T, int K, const bf16* __restrict__ w,
                                    long long ldw, int N,
                                    const float* __restrict__ bias, int act,
                                    int mode, float alpha, void* out,
                                    long long ldo) {
  griddep_wait();
  griddep_launch_dependents();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= T * N) return;
  const int t = gw / N, n = gw % N;
  const float* xr = x + (long long)t * ldx;
  const bf16* wr = w + (long long)n * ldw;
  float acc = 0.f;
  for (int k = lane; k < K; k += 32) acc += xr[k] * __bfloat162float(wr[k]);
  acc = warp_sum(acc);
  if (lane == 0) {
    float y = acc + (bias ? bias[n] : 0.f);
    if (act == FVB_ACT_SILU) y = silu_f(y);
    else if (act == FVB_ACT_GELU_TANH) y = gelu_tanh_f(y);
    if (mode == 0)
      reinterpret_cast<float*>(out)[(long long)t * ldo + n] = y;
    else if (mode == 1)
      reinterpret_cast<bf16*>(out)[(long long)t * ldo + n] =
          __float2bfloat16(y);
    else
      reinterpret_cast<float*>(out)[(long long)t * ldo + n] += alpha * y;
  }
}


__device__ __forceinline__ float small_linear_finish(float acc, const float* bias,
                                                     int n, int act) {
  float y = acc + (bias ? bias[n] : 0.f);
  if (act == FVB_ACT_SILU) y = silu_f(y);
  else if (act == FVB_ACT_GELU_TANH) y = gelu_tanh_f(y);
  return y;
}

__device__ __forceinline__ void small_linear_store(void* out, long long ldo, int t,
                                                   int n, int mode, float alpha,
                                                   float y) {
  if (mode == 0)
    reinterpret_cast<float*>(out)[(long long)t * ldo + n] = y;
  else if (mode == 1)
    reinterpret_cast<bf16*>(out)[(long long)t * ldo + n] = __float2bfloat16(y);
  else
    reinterpret_cast<float*>(out)[(long long)t * ldo + n] += alpha * y;
}

// Narrow K (<= 64, multiple of 8; the action / state input projections):
// one thread per output, the weight row read as 16-byte vectors, the token
// row staged once per block in shared memory.  Block = one token x 256
// outputs.
__global__ void __launch_bounds__(256)
    small_linear_narrow_kernel(const float* __restrict__ x, long long ldx, int K,
                               const bf16* __restrict__ w, long long ldw, int N,
                               const float* __restrict__ bias, int act, int mode,
                               float alpha, void* out, long long ldo) {
  __shared__ float xs[64];
  griddep_wait();
  griddep_launch_dependents();
  const int chunks = (N + 255) / 256;
  const int t = blockIdx.x / chunks;
  const int n = (blockIdx.x % chunks) * 256 + threadIdx.x;
  if (threadIdx.x < K) xs[threadIdx.x] = x[(long long)t * ldx + threadIdx.x];
  __syncthreads();
  if (n >= N) return;
  const uint4* wr = reinterpret_cast<const uint4*>(w + (long long)n * ldw);
  float acc = 0.f;
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    if (c * 8 >= K) break;
    const uint4 q = __ldg(wr + c);
    const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wd[e]));
      acc += xs[c * 8 + 2 * e] * f.x + xs[c * 8 + 2 * e + 1] * f.y;
    }
  }
  small_linear_store(out, ldo, t, n, mode, alpha, small_linear_finish(acc, bias, n, act));
}

// Wide K (multiple of 256, <= 4096; the action output projection): one warp
// per output, every lane loading 16-byte weight vectors and two float4 of
// the token row per 256-wide step, all steps' loads in flight together.
__global__ void __launch_bounds__(256)
    small_linear_wide_kernel(const float* __restrict__ x, long long ldx, int T,
                             int K, const bf16* __restrict__ w, long long ldw,
                             int N, const float* __restrict__ bias, int act,
                             int mode, float alpha, void* out, long long ldo) {
  griddep_wait();
  griddep_launch_dependents();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (gw >= T * N) return;
  const int t = gw / N, n = gw % N;
  const float* xr = x + (long long)t * ldx + lane * 8;
  const bf16* wr = w + (long long)n * ldw + lane * 8;
  float acc = 0.f;
#pragma unroll 4
  for (int k = 0; k < K; k += 256) {
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(wr + k));
    const float4 a = *reinterpret_cast<const float4*>(xr + k);
    const float4 b = *reinterpret_cast<const float4*>(xr + k + 4);
    const float2 w0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.x));
    const float2 w1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.y));
    const float2 w2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.z));
    const float2 w3 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.w));
    acc += a.x * w0.x + a.y * w0.y + a.z * w1.x + a.w * w1.y +
           b.x * w2.x + b.y * w2.y + b.z * w3.x + b.w * w3.y;
  }
  acc = warp_sum(acc);
  if (lane == 0)
    small_linear_store(out, ldo, t, n, mode, alpha, small_linear_finish(acc, bias, n, act));
}

// Failure-path probe: one thread waits on an mbarrier that nothing arrives
// on, through the same bounded wait as every kernel here, with a short
// limit; the wait gives up, records FVB_ERR_DEVICE_TIMEOUT in the status
// word and the kernel returns normally (the context stays usable).
__device__ int g_probe_result;
__global__ void wait_timeout_probe_kernel(unsigned long long limit_ns, int* gave_up) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  fence_barrier_init();
  const bool ok = mbar_wait_limit(&bar, 0, limit_ns);
  *gave_up = ok ? 0 : 1;
}


// ---------------------------------------------------------------------------
// Norms of bf16 rows (fvb_norm_bf16): one warp per row, 8 values per lane
// per step (16-byte loads); LayerNorm takes a second pass for the centred
// variance as the reference kernel does.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void unpack8(const uint4 q, float (&v)[8]) {
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[e]));
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}

__global__ void __launch_bounds__(256)
    norm_bf16_kernel(int mode, const bf16* __restrict__ x, long long ld_in,
                     bf16* __restrict__ out, long long ld_out, int rows, int dim,
                     const bf16* __restrict__ w, const bf16* __restrict__ b,
                     const bf16* __restrict__ style, bf16* __restrict__ gate_out,
                     long long ld_gate, float eps) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const bf16* xr = x + (long long)row * ld_in;
  float s = 0.f, ss = 0.f;
  for (int c = lane * 8; c < dim; c += 256) {
    float v[8];
    unpack8(*reinterpret_cast<const uint4*>(xr + c), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) { s += v[e]; ss += v[e] * v[e]; }
  }
  s = warp_sum(s);
  ss = warp_sum(ss);
  float mean = 0.f, rstd;
  if (mode == FVB_NORM_LAYER) {
    mean = s / dim;
    float vs = 0.f;
    for (int c = lane * 8; c < dim; c += 256) {
      float v[8];
      unpack8(*reinterpret_cast<const uint4*>(xr + c), v);
#pragma unroll
      for (int e = 0; e < 8; ++e) vs += (v[e] - mean) * (v[e] - mean);
    }
    rstd = rsqrtf(warp_sum(vs) / dim + eps);
  } else {
    rstd = rsqrtf(ss / dim + eps);
  }
  bf16* orow = out + (long long)row * ld_out;
  for (int c = lane * 8; c < dim; c += 256) {
    float v[8], y[8];
    unpack8(*reinterpret_cast<const uint4*>(xr + c), v);
#pragma unroll
    for (int e = 0; e < 8; ++e) y[e] = (v[e] - mean) * rstd;
    if (mode == FVB_NORM_LAYER) {
      float wv[8], bv[8];
      unpack8(*reinterpret_cast<const uint4*>(w + c), wv);
      unpack8(*reinterpret_cast<const uint4*>(b + c), bv);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = y[e] * wv[e] + bv[e];
    } else if (mode == FVB_NORM_ADA_STYLE) {
      float sc[8], sh[8];
      unpack8(*reinterpret_cast<const uint4*>(style + c), sc);
      unpack8(*reinterpret_cast<const uint4*>(style + dim + c), sh);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = y[e] * (1.f + sc[e]) + sh[e];
      *reinterpret_cast<uint4*>(gate_out + (long long)row * ld_gate + c) =
          *reinterpret_cast<const uint4*>(style + 2 * dim + c);
    }
    *reinterpret_cast<uint4*>(orow + c) =
        make_uint4(pack_bf16x2(y[0], y[1]), pack_bf16x2(y[2], y[3]),
                   pack_bf16x2(y[4], y[5]), pack_bf16x2(y[6], y[7]));
  }
}


// ---------------------------------------------------------------------------
// Row softmax of materialised attention logits (fvb_softmax_rows): f32
// logits [rows, keys] -> bf16 probabilities.  Key j takes part when
// j >= n_prefix (suffix keys) or j < min(valid_prefix, n_prefix); masked
// keys hold the reference's large negative value, so a row with every key
// masked comes out uniform as in the reference kernels.  One warp per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
    softmax_rows_kernel(const float* __restrict__ in, long long ld_in, int rows,
                        int keys, int n_prefix, const int* __restrict__ valid_prefix,
                        bf16* __restrict__ out, long long ld_out) {
  griddep_wait();
  griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float big_neg = -2.3819763e38f;
  const int vl = max(0, min(*valid_prefix, n_prefix));
  const float* x = in + (long long)row * ld_in;
  float mx = big_neg;
  for (int j = lane; j < keys; j += 32) {
    const bool ok = j >= n_prefix || j < vl;
    mx = fmaxf(mx, ok ? x[j] : big_neg);
  }
  mx = warp_max(mx);
  float sum = 0.f;
  for (int j = lane; j < keys; j += 32) {
    const bool ok = j >= n_prefix || j < vl;
    sum += __expf((ok ? x[j] : big_neg) - mx);
  }
  sum = warp_sum(sum);
  const float inv = 1.f / sum;
  bf16* o = out + (long long)row * ld_out;
  for (int j = lane; j < keys; j += 32) {
    const bool ok = j >= n_prefix || j < vl;
    o[j] = __float2bfloat16(__expf((ok ? x[j] : big_neg) - mx) * inv);
  }
}

}  // namespace fvb

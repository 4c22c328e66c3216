// misc.cu — layout kernels: strided staging copies, memset_d32, the
// reference-exact single-channel im2col / col2im (remora/runtime.py:1274-1305)
// and the rank-2 transpose (remora/runtime.py:1052-1056, VJP remora/ad.py:113).
#include <algorithm>

#include "common.cuh"

namespace remora {

namespace {

struct StridedView {
  int64_t shape[REMORA_MAX_RANK];
  int64_t stride[REMORA_MAX_RANK];
  int32_t rank;
};

template <typename T, bool kToContig>
__global__ void __launch_bounds__(256) strided_copy_kernel(const T *__restrict__ src, T *__restrict__ dst,
                                                           StridedView v, int64_t n) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    int64_t rem = i, off = 0;
    for (int d = v.rank - 1; d >= 0; --d) {
      const int64_t q = rem % v.shape[d];
      rem /= v.shape[d];
      off += q * v.stride[d];
    }
    if (kToContig) dst[i] = src[off];
    else dst[off] = src[i];
  }
}

StridedView make_view(const DescView &d) {
  StridedView v{};
  v.rank = d.rank;
  for (int i = 0; i < d.rank; ++i) {
    v.shape[i] = d.sizes[i];
    v.stride[i] = d.strides[i];
  }
  return v;
}

int grid_for(int64_t n, int sm_count) {
  return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sm_count * 16));
}

__global__ void memset32_kernel(uint32_t *dst, uint32_t value, int64_t count) {
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += step) dst[i] = value;
}

// cols[(i*ow + j)*kh*kw + a*kw + b] = img[(i*s + a)*W + (j*s + b)], with the
// image and the patch matrix addressed through their descriptor strides.
__global__ void __launch_bounds__(256) im2col_kernel(const float *__restrict__ img, int64_t is0, int64_t is1,
                                                     float *__restrict__ cols, int64_t cs0, int64_t cs1,
                                                     int64_t oh, int64_t ow, int kh, int kw, int stride) {
  const int64_t n = oh * ow * kh * kw;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += step) {
    const int64_t col = t % (kh * kw), patch = t / (kh * kw);
    const int64_t i = patch / ow, j = patch % ow;
    const int a = (int)(col / kw), b = (int)(col % kw);
    cols[patch * cs0 + col * cs1] = img[(i * stride + a) * is0 + (j * stride + b) * is1];
  }
}

// Gather form of the overlap-add: each image pixel sums, in patch order,
// every column entry that covers it (no atomics, deterministic).  The sum is
// kept in f64 and rounded once, as the reference accumulates into a float64
// image before coercing it to f32 (remora/runtime.py:1300-1305).
__global__ void __launch_bounds__(256) col2im_kernel(const float *__restrict__ cols, int64_t cs0, int64_t cs1,
                                                     float *__restrict__ img, int64_t is0, int64_t is1,
                                                     int64_t H, int64_t W, int64_t oh, int64_t ow, int kh,
                                                     int kw, int stride) {
  const int64_t n = H * W;
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += step) {
    const int64_t y = t / W, x = t % W;
    double acc = 0.0;
    for (int64_t i = 0; i < oh; ++i) {
      const int64_t a = y - i * stride;
      if (a < 0) break;
      if (a >= kh) continue;
      for (int64_t j = 0; j < ow; ++j) {
        const int64_t b = x - j * stride;
        if (b < 0) break;
        if (b >= kw) continue;
        acc = __dadd_rn(acc, (double)cols[(i * ow + j) * cs0 + (a * kw + b) * cs1]);
      }
    }
    img[y * is0 + x * is1] = (float)acc;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) transpose_kernel(const T *__restrict__ in, int64_t is0, int64_t is1,
                                                        T *__restrict__ out, int64_t os0, int64_t os1,
                                                        int64_t R, int64_t C) {
  __shared__ T tile[32][33];
  for (int64_t r0 = (int64_t)blockIdx.y * 32; r0 < R; r0 += (int64_t)gridDim.y * 32)
    for (int64_t c0 = (int64_t)blockIdx.x * 32; c0 < C; c0 += (int64_t)gridDim.x * 32) {
      for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int64_t r = r0 + k, c = c0 + threadIdx.x;
        if (r < R && c < C) tile[k][threadIdx.x] = in[r * is0 + c * is1];
      }
      __syncthreads();
      for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int64_t c = c0 + k, r = r0 + threadIdx.x;
        if (r < R && c < C) out[c * os0 + r * os1] = tile[threadIdx.x][k];
      }
      __syncthreads();
    }
}

}  // namespace

int copy_to_contiguous(const DescView &src, int esize, void *dst, cudaStream_t stream, int sm_count) {
  const int64_t n = src.numel();
  if (n == 0) return REMORA_OK;
  StridedView v = make_view(src);
  note_launch();
  if (esize == 4)
    strided_copy_kernel<uint32_t, true><<<grid_for(n, sm_count), 256, 0, stream>>>(
        (const uint32_t *)src.data(4), (uint32_t *)dst, v, n);
  else
    strided_copy_kernel<uint8_t, true><<<grid_for(n, sm_count), 256, 0, stream>>>(
        (const uint8_t *)src.data(1), (uint8_t *)dst, v, n);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int copy_from_contiguous(const void *src, const DescView &dst, int esize, cudaStream_t stream, int sm_count) {
  const int64_t n = dst.numel();
  if (n == 0) return REMORA_OK;
  StridedView v = make_view(dst);
  note_launch();
  if (esize == 4)
    strided_copy_kernel<uint32_t, false><<<grid_for(n, sm_count), 256, 0, stream>>>(
        (const uint32_t *)src, (uint32_t *)dst.data(4), v, n);
  else
    strided_copy_kernel<uint8_t, false><<<grid_for(n, sm_count), 256, 0, stream>>>(
        (const uint8_t *)src, (uint8_t *)dst.data(1), v, n);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

}  // namespace remora

using namespace remora;

extern "C" {

int remora_b200_memset_d32(RemoraB200Ctx *ctx, void *dst, uint32_t value, size_t count,
                           remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (count == 0) return REMORA_OK;
  if (dst == nullptr || (reinterpret_cast<uintptr_t>(dst) & 3))
    return fail(REMORA_ERR_ARG, "memset_d32: null or unaligned destination");
  note_launch();
  memset32_kernel<<<grid_for((int64_t)count, ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (uint32_t *)dst, value, (int64_t)count);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

static int check_im2col(const RemoraIm2colSpec *spec, int64_t H, int64_t W) {
  if (spec == nullptr) return fail(REMORA_ERR_ARG, "im2col: null spec");
  if (spec->kh < 1 || spec->kw < 1 || spec->stride < 1)
    return fail(REMORA_ERR_ARG, "im2col: kernel %dx%d stride %d", spec->kh, spec->kw, spec->stride);
  if (spec->kh > H || spec->kw > W)
    return fail(REMORA_ERR_SHAPE, "im2col: kernel %dx%d larger than the %lldx%lld image", spec->kh,
                spec->kw, (long long)H, (long long)W);
  return REMORA_OK;
}

int remora_b200_im2col(RemoraB200Ctx *ctx, const RemoraIm2colSpec *spec, const RemoraMemRef2 *image,
                       RemoraMemRef2 *cols, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView im, co;
  REMORA_TRY(read_desc(image, 2, &im, "im2col image"));
  REMORA_TRY(read_desc(cols, 2, &co, "im2col columns"));
  REMORA_TRY(check_im2col(spec, im.sizes[0], im.sizes[1]));
  const int64_t oh = (im.sizes[0] - spec->kh) / spec->stride + 1;
  const int64_t ow = (im.sizes[1] - spec->kw) / spec->stride + 1;
  if (co.sizes[0] != oh * ow || co.sizes[1] != (int64_t)spec->kh * spec->kw)
    return fail(REMORA_ERR_SHAPE, "im2col: columns must be [%lld, %d]", (long long)(oh * ow),
                spec->kh * spec->kw);
  const int64_t n = co.numel();
  if (n == 0) return REMORA_OK;
  note_launch();
  im2col_kernel<<<grid_for(n, ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (const float *)im.data(4), im.strides[0], im.strides[1], (float *)co.data(4), co.strides[0],
      co.strides[1], oh, ow, spec->kh, spec->kw, spec->stride);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_col2im(RemoraB200Ctx *ctx, const RemoraIm2colSpec *spec, const RemoraMemRef2 *cols,
                       RemoraMemRef2 *image, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView im, co;
  REMORA_TRY(read_desc(cols, 2, &co, "col2im columns"));
  REMORA_TRY(read_desc(image, 2, &im, "col2im image"));
  REMORA_TRY(check_im2col(spec, im.sizes[0], im.sizes[1]));
  const int64_t oh = (im.sizes[0] - spec->kh) / spec->stride + 1;
  const int64_t ow = (im.sizes[1] - spec->kw) / spec->stride + 1;
  if (co.sizes[0] != oh * ow || co.sizes[1] != (int64_t)spec->kh * spec->kw)
    return fail(REMORA_ERR_SHAPE, "col2im: columns must be [%lld, %d]", (long long)(oh * ow),
                spec->kh * spec->kw);
  const int64_t n = im.numel();
  if (n == 0) return REMORA_OK;
  note_launch();
  col2im_kernel<<<grid_for(n, ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (const float *)co.data(4), co.strides[0], co.strides[1], (float *)im.data(4), im.strides[0],
      im.strides[1], im.sizes[0], im.sizes[1], oh, ow, spec->kh, spec->kw, spec->stride);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_transpose(RemoraB200Ctx *ctx, int32_t dtype, const RemoraMemRef2 *in, RemoraMemRef2 *out,
                          remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView a, b;
  REMORA_TRY(read_desc(in, 2, &a, "transpose input"));
  REMORA_TRY(read_desc(out, 2, &b, "transpose output"));
  if (b.sizes[0] != a.sizes[1] || b.sizes[1] != a.sizes[0])
    return fail(REMORA_ERR_SHAPE, "transpose: output must be [%lld, %lld]", (long long)a.sizes[1],
                (long long)a.sizes[0]);
  const int64_t R = a.sizes[0], C = a.sizes[1];
  if (R == 0 || C == 0) return REMORA_OK;
  dim3 block(32, 8);
  dim3 grid((unsigned)std::min<int64_t>((C + 31) / 32, 65535), (unsigned)std::min<int64_t>((R + 31) / 32, 65535));
  const int es = dtype_size(dtype);
  if (es != 4 && es != 1) return fail(REMORA_ERR_ARG, "transpose: bad dtype %d", dtype);
  note_launch();
  if (es == 4)
    transpose_kernel<uint32_t><<<grid, block, 0, (cudaStream_t)stream>>>(
        (const uint32_t *)a.data(4), a.strides[0], a.strides[1], (uint32_t *)b.data(4), b.strides[0],
        b.strides[1], R, C);
  else
    transpose_kernel<uint8_t><<<grid, block, 0, (cudaStream_t)stream>>>(
        (const uint8_t *)a.data(1), a.strides[0], a.strides[1], (uint8_t *)b.data(1), b.strides[0],
        b.strides[1], R, C);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

}  // extern "C"

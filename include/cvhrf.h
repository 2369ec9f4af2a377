/*
 * cvhrf.h — C ABI of the B200 (sm_100a) wave-optics hot path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (``cudaStream_t`` passed as ``void*``), never allocates device memory in the
 * data path (scratch comes from a caller-provided workspace whose size is given
 * by the matching ``*_workspace_bytes`` query), and returns an ``int`` status
 * (``CVHRF_OK`` == 0).  Complex data are complex64 interleaved (re, im) — the
 * memory layout of ``torch.complex64``.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   - propagation: cuda_prop/python_function.py:109-218 (BandlimitedPropagationFunction
 *     forward/backward = zero_pad -> fft2 -> fftshift -> transfer kernel -> ifftshift ->
 *     ifft2 -> crop) and the kernels it calls, cuda_prop/cpp/bandlimited_propagation.cpp:34-79,
 *     cuda_prop/cuda/bandlimited_propagation_cuda.cu:29-274; the plane/channel loop that
 *     sums planes, model.py:1251-1272.
 *   - rasterizer: cuda_prop/cov3d_cuda/python_import.py:283-342 (SplatTileCuda) ->
 *     binding.cpp:31-36 (Rasterizer.forward/backward) ->
 *     wave_rasterizer/rasterizer_splat.cu:325-684.
 *   - sparse Adam: cuda_prop/cov3d_cuda/python_import.py:457-460 (sparse_adam_update) ->
 *     conv.cu:1230-1246 (adamUpdate) and utils/optimizer.py:180-265 (SparseGaussianAdam.step).
 */
#ifndef CVHRF_H_
#define CVHRF_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------------- */
#define CVHRF_OK 0
#define CVHRF_EINVAL 1        /* bad argument (null pointer, size, unsupported shape)   */
#define CVHRF_EWORKSPACE 2    /* workspace too small                                     */
#define CVHRF_ECUDA 3         /* a CUDA runtime call failed (see cvhrf_last_cuda_error)  */
#define CVHRF_EUNSUPPORTED 4  /* size outside what the kernels are built for             */

/* Human-readable text for a status code (static storage). */
const char* cvhrf_status_string(int status);
/* The cudaError_t of the last failing CUDA call made by this library on this thread. */
int cvhrf_last_cuda_error(void);
/* Library version, e.g. 100 for 0.1.0. */
int cvhrf_version(void);

/* ---- band-limited angular-spectrum propagation ---------------------------- */
/*
 * A plan holds the twiddle and digit-reversal tables for one padded size
 * P = 2*S on one device (created once, like an FFT plan).  S must factor into
 * 2, 3 and 5 only, 8 <= S <= 4096.
 * Replaces: the cuFFT plans behind torch.fft.fft2/ifft2 (python_function.py:129-161).
 */
typedef struct cvhrf_asm_plan cvhrf_asm_plan;
int cvhrf_asm_plan_create(int S, cvhrf_asm_plan** plan_out);
int cvhrf_asm_plan_destroy(cvhrf_asm_plan* plan);

/*
 * Workspace bytes for propagating `items` inputs of Hi x Wi to `out_items` outputs
 * of Ho x Wo with padded grid 2S x 2S (an intermediate of items*Hi*2S and one of
 * out_items*Ho*2S complex64 values, 256-byte aligned).
 */
size_t cvhrf_asm_workspace_bytes(int S, int items, int Hi, int Wi, int out_items, int Ho, int Wo);

/*
 * One propagation (python_function.py:109-163 forward; :165-218 backward):
 *   out = crop_{Ho x Wo}( IFFT2( H_{lambda,d} * A * FFT2( pad_{2S x 2S}(in) ) ) )
 * with H = exp(i d kz) band-limited (bandlimited_propagation_cuda.cu:29-86) and A the
 * circular aperture of radius `aperture` in fftshifted index space (disabled if <= 0).
 * Forward: in = field (Hi x Wi), Ho = Wo = S.  The reference's backward equals this
 * call with in = grad (S x S), out = grad_field (Hi x Wi) and distance -> -distance.
 * accumulate != 0 adds into `out` instead of overwriting it.
 */
int cvhrf_asm_propagate(const cvhrf_asm_plan* plan,
                        const void* in, int Hi, int Wi,
                        void* out, int Ho, int Wo,
                        float wavelength, float pixel_pitch, float distance, float aperture,
                        int accumulate,
                        void* workspace, size_t workspace_bytes, void* stream);

/*
 * K planes x C channels in one call, summed over planes (model.py:1251-1272):
 *   holo[c] = sum_p propagate(fields[p, c], wavelengths[c], distances[p])
 * fields: K x C x H x W complex64; holo: C x S x S complex64.
 * wavelengths (C) and distances (K) are HOST arrays; `distances` are the signed
 * propagation distances as passed to BandlimitedPropagation (model.py:1259: -d_p).
 */
int cvhrf_asm_propagate_planes(const cvhrf_asm_plan* plan,
                               const void* fields, int K, int C, int H, int W,
                               const float* wavelengths, const float* distances,
                               float pixel_pitch, float aperture,
                               void* holo,
                               void* workspace, size_t workspace_bytes, void* stream);

/*
 * Adjoint of cvhrf_asm_propagate_planes (the backward of the summed propagation):
 *   grad_fields[p, c] = propagate(grad_holo[c], wavelengths[c], -distances[p]) cropped to H x W
 * grad_holo: C x S x S; grad_fields: K x C x H x W.
 */
int cvhrf_asm_propagate_planes_adjoint(const cvhrf_asm_plan* plan,
                                       const void* grad_holo, int K, int C, int H, int W,
                                       const float* wavelengths, const float* distances,
                                       float pixel_pitch, float aperture,
                                       void* grad_fields,
                                       void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CVHRF_H_ */

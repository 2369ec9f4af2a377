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
/* Number of CUDA kernels this library has launched in this process (diagnostics;
 * no counterpart in the reference). */
unsigned long long cvhrf_kernel_launch_count(void);

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

/*
 * Precomputed transfer tables for cvhrf_asm_propagate_planes and its adjoint.
 * The transfer function x aperture of every (plane p, channel c) depends only on
 * (S, wavelength, distance, pitch, aperture), which stay fixed across a training
 * run, so it can be evaluated once (same values as the per-call evaluation) and
 * read back by the column pass.  A table holds K*C items of (2S)^2 complex64 values
 * in the column pass's order (item p*C + c); only sizes with a compile-time FFT
 * plan (S = 64, 128, 256, 384, 512, 800, 1024, 1920, 2048) are supported, and
 * K*C <= 64.  cvhrf_asm_transfer_table_bytes returns 0 for unsupported arguments.
 * The table-based calls take the same fields / holo / workspace as
 * cvhrf_asm_propagate_planes(_adjoint); with a table the column pass makes K
 * forward and one inverse column transform per channel (the spectra of the K
 * planes are summed before the inverse transform), and the adjoint one forward and
 * K inverse ones (it uses conj(H), the transfer function of distance -d).
 * No counterpart in the reference, whose BandlimitedPropagation evaluates the
 * transfer function in every call (bandlimited_propagation_cuda.cu:29-86).
 */
size_t cvhrf_asm_transfer_table_bytes(int S, int K, int C);
int cvhrf_asm_transfer_table_build(const cvhrf_asm_plan* plan, int K, int C,
                                   const float* wavelengths, const float* distances,
                                   float pixel_pitch, float aperture, void* table, void* stream);
/*
 * A table from a caller-supplied transfer function instead of the built-in one: `centred`
 * holds `items` (= K*C, item p*C + c) complex64 arrays of (2S)^2 values in centred
 * (fftshifted) order, row-major, element [y][x] applying to the spectrum bin that
 * torch.fft.fftshift moves to (y, x); the aperture, if any, is already multiplied in.
 * This is how a propagator whose kernel comes from elsewhere (odak's
 * get_propagation_kernel, utils/propagator.py:480-517, cached in self.kernels) runs on
 * these column passes.  The planes call multiplies by the table; the adjoint call by its
 * conjugate.
 */
int cvhrf_asm_transfer_table_upload(const cvhrf_asm_plan* plan, int items, const void* centred, void* table,
                                    void* stream);
int cvhrf_asm_propagate_planes_table(const cvhrf_asm_plan* plan,
                                     const void* fields, int K, int C, int H, int W,
                                     const void* table, void* holo,
                                     void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_asm_propagate_planes_adjoint_table(const cvhrf_asm_plan* plan,
                                             const void* grad_holo, int K, int C, int H, int W,
                                             const void* table, void* grad_fields,
                                             void* workspace, size_t workspace_bytes, void* stream);

/*
 * cvhrf_asm_propagate without any device allocation and without a plan.
 * No counterpart in the reference: it exists for callers that cannot allocate
 * device memory when they propagate (a frozen or exhausted memory pool, a plugin
 * host that forbids allocation inside its execute callback, a real-time loop that
 * must not touch the allocator).  Its scratch — two intermediate spectra and the
 * FFT tables — is one fixed device array inside the library (about 8.2 MB, kept
 * by every GPU that loads the library until the process exits), so S is limited
 * to 8 <= S <= 512 (larger S returns CVHRF_EUNSUPPORTED).  Same arguments and
 * result as cvhrf_asm_propagate otherwise.  The first call on a device looks up
 * that array's device address (with the device current); make that first call
 * before any stream capture.  All calls share the array and overwrite it, so calls
 * that overlap on the GPU race: order them on one stream.  The looked-up address is
 * kept for the life of the process, so do not call it again on a device after
 * cudaDeviceReset (or any other reset of that device's primary context).
 */
int cvhrf_asm_propagate_noalloc(const void* in, int Hi, int Wi, void* out, int Ho, int Wo, int S,
                                float wavelength, float pixel_pitch, float distance, float aperture,
                                int accumulate, void* stream);


/* ---- complex-field tile rasterizer ---------------------------------------- */
/*
 * Inputs of SplatTileCuda.forward (python_import.py:283-313), all float32 device
 * arrays, contiguous: cam_means N x 3, z_vals N, quats N x 4, scales N x 3,
 * colours N x C, phase N x C, opacities N, plane_probs N x K, view_matrix 3 x 3
 * (row-major).  C <= 3 (MAX_CHANNELS), K <= 8 (MAX_PLANES); tiles are 16 x 16.
 */
typedef struct {
  int N, K, C, W, H;
  float fx, fy, px, py, near_plane, far_plane;
  const float* cam_means;
  const float* z_vals;
  const float* quats;
  const float* scales;
  const float* colours;
  const float* phase;
  const float* opacities;
  const float* plane_probs;
  const float* view_matrix;
} cvhrf_raster_scene;

/*
 * Forward, phase 1 (replaces rasterizer_splat.cu:363-432: markVisible, means2d,
 * cov2d, preprocessGaussiansKernel, CUB scan): per-Gaussian projection, radius and
 * tile count, depth-key sort, pair offsets.  Writes counts_dev[0] = number of
 * (tile, Gaussian) pairs and counts_dev[1] = number of visible Gaussians (device
 * int32[2]).  `geom_ws` must stay untouched until the backward has run.
 */
size_t cvhrf_raster_geometry_workspace_bytes(int N, int K, int C);
int cvhrf_raster_forward_geometry(const cvhrf_raster_scene* scene, void* geom_ws, size_t geom_bytes,
                                  int32_t* counts_dev, void* stream);

/*
 * Forward, phase 2 (replaces rasterizer_splat.cu:435-548: duplicateWithKeys, CUB
 * radix sort, identifyTileRanges, renderTileKernel): emits and stably sorts the
 * pairs, renders all K planes in one pass per tile.  Outputs (device):
 *   field K x C x H x W complex64; final_Ts K x H x W f32; n_contrib K x H x W i32;
 *   point_list num_pairs i32; ranges (tiles x 2) i32; visible_indices num_visible i64.
 * `bin_ws` must stay untouched until the backward has run.
 */
size_t cvhrf_raster_binning_workspace_bytes(int N, int num_pairs, int W, int H);
int cvhrf_raster_forward_render(const cvhrf_raster_scene* scene, const void* geom_ws, size_t geom_bytes,
                                int num_pairs, int num_visible, void* bin_ws, size_t bin_bytes,
                                void* field, float* final_Ts, int32_t* n_contrib, int32_t* point_list,
                                int32_t* ranges, int64_t* visible_indices, void* stream);

/*
 * Forward phase 2 without the host round trip (for CUDA-graph capture): identical
 * outputs, but the pair count stays on the device (counts_dev[0] from
 * cvhrf_raster_forward_geometry), point_list / the binning workspace are sized for
 * pairs_capacity, visibility is returned as a per-Gaussian uint8 mask (N) instead of
 * compacted indices, and *overflow (device int32, caller-zeroed) is set to 1 when the
 * count exceeds the capacity -- then nothing is rendered and the call must be repeated
 * with a larger capacity.  The backward takes num_pairs = pairs_capacity.
 */
int cvhrf_raster_forward_render_capacity(const cvhrf_raster_scene* scene, const void* geom_ws, size_t geom_bytes,
                                         const int32_t* counts_dev, int pairs_capacity, void* bin_ws,
                                         size_t bin_bytes, void* field, float* final_Ts, int32_t* n_contrib,
                                         int32_t* point_list, int32_t* ranges, uint8_t* visible_mask,
                                         int32_t* overflow, void* stream);

/*
 * Backward (replaces rasterizer_splat.cu:551-684, renderBackwardTileKernel and the
 * geometry backward): atomic-free — each tile writes one gradient record per
 * (tile, Gaussian) pair, then one thread per Gaussian reduces its records and
 * chains them through the projection.  grad_field: K x C x H x W complex64.
 * Gradient outputs are dense N x {3,1,4,3,C,C,1,K} float32 (grad_z_vals is all 0
 * as in the reference).
 */
size_t cvhrf_raster_backward_workspace_bytes(int num_pairs, int K, int C);
int cvhrf_raster_backward(const cvhrf_raster_scene* scene, const void* geom_ws, size_t geom_bytes,
                          const void* bin_ws, size_t bin_bytes, int num_pairs,
                          const void* grad_field, const float* final_Ts, const int32_t* n_contrib,
                          const int32_t* point_list, const int32_t* ranges, void* bwd_ws, size_t bwd_bytes,
                          float* grad_cam_means, float* grad_z_vals, float* grad_quats, float* grad_scales,
                          float* grad_colours, float* grad_phase, float* grad_opacities,
                          float* grad_plane_probs, void* stream);

/* ---- sparse Adam ----------------------------------------------------------- */
/*
 * One parameter group: param / exp_avg / exp_avg_sq / grad are dense N x D float32
 * (device).  Sparse groups update the rows listed in `visible`; dense groups (the
 * reference's 1-D parameters, utils/optimizer.py:207-217) update all N rows.
 */
typedef struct {
  float* param;
  const float* grad;
  float* exp_avg;
  float* exp_avg_sq;
  int N, D;
  int dense;
  float lr, eps;
} cvhrf_adam_group;

/*
 * All groups in one launch (replaces conv.cu:1230-1246 adamUpdate, called once per
 * group by SparseGaussianAdam.step, utils/optimizer.py:219-253; the gathered
 * (B, V, D) gradient copy is not needed — dense gradient rows are read in place).
 * visible: V int64 row indices (device).  At most 16 groups.
 */
int cvhrf_sparse_adam(const cvhrf_adam_group* groups, int ngroups, const int64_t* visible, int V,
                      float beta1, float beta2, void* stream);
/*
 * The same update with the visible rows given as a row mask (uint8, mask_len rows,
 * non-zero = update; dense groups ignore it).  Rows are streamed in memory order.
 * cvhrf_rows_to_mask builds such a mask from row indices (zeroes it first).
 */
int cvhrf_sparse_adam_masked(const cvhrf_adam_group* groups, int ngroups, const uint8_t* mask, int mask_len,
                             float beta1, float beta2, void* stream);
int cvhrf_rows_to_mask(const int64_t* rows, int V, uint8_t* mask, int mask_len, void* stream);

/* ---- fused SSIM (the training loss's SSIM term) ------------------------------ */
/*
 * SSIM map of img1 against img2 (C x H x W float32 each, device) with an 11 x 11
 * Gaussian window (sigma 1.5), zero padding outside the image, constants C1, C2
 * (the reference uses 0.01^2 and 0.03^2).  Replaces fusedssim / fusedssim_backward
 * (conv.cu:935-1195) behind FusedSSIMMap / fast_ssim (python_import.py:43-57, 449-454).
 * cvhrf_ssim_forward writes the map (if map != NULL) and/or its mean (if mean != NULL,
 * a DEVICE float), and leaves in the workspace what the backward needs.
 * cvhrf_ssim_backward: gradient with respect to img1 for an upstream gradient given
 * either per pixel (dL_dmap) or for the mean (dL_dmean, a DEVICE float); exactly one of
 * the two.  The workspace must be the one the matching forward filled.
 */
size_t cvhrf_ssim_workspace_bytes(int C, int H, int W);
int cvhrf_ssim_forward(const float* img1, const float* img2, int C, int H, int W, float C1, float C2,
                       float* map, float* mean, void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_ssim_backward(const float* img1, const float* img2, int C, int H, int W,
                        const float* dL_dmap, const float* dL_dmean, float* grad_img1,
                        const void* workspace, size_t workspace_bytes, void* stream);

/* ---- Adan (the optimizer of the reference's training script) -------------- */
/*
 * One launch for every group (replaces Adan.step, utils/optimizer.py:374-484, with its
 * foreach kernels :545-611).  The per-step scalars are the caller's and are the ones the
 * reference hands to torch (computed in double, each rounded to float once):
 * beta1..3; one_minus_beta1..3 = 1 - beta; bias_correction3_sqrt = sqrt(1 - beta3^step);
 * step_size = lr / (1 - beta1^step); step_size_diff = lr beta2 / (1 - beta2^step);
 * decay = 1 - lr wd (no_prox) or 1 + lr wd (otherwise).
 * first_step = 1 on a group's first step (neg_pre_grad is then taken as -grad).
 * clip: DEVICE float global-norm clip factor, or NULL for 1 (cvhrf_adan_clip_factor
 * computes it without a host round trip: min(max_grad_norm / (||all grads|| + eps), 1)).
 * grad is scaled in place by the clip factor, as the reference's grad.mul_ does.
 * The clip workspace must be zeroed once (cvhrf_adan_clip_init_workspace).  At most 16 groups.
 */
typedef struct {
  float* param;
  float* grad;
  float* exp_avg;
  float* exp_avg_sq;
  float* exp_avg_diff;
  float* neg_pre_grad;
  long long n;
  float beta1, beta2, beta3, one_minus_beta1, one_minus_beta2, one_minus_beta3;
  float bias_correction3_sqrt, eps, step_size, step_size_diff, decay;
  int no_prox, first_step;
} cvhrf_adan_group;
int cvhrf_adan(const cvhrf_adan_group* groups, int ngroups, const float* clip, void* stream);
size_t cvhrf_adan_clip_workspace_bytes(void);
int cvhrf_adan_clip_init_workspace(void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_adan_clip_factor(const cvhrf_adan_group* groups, int ngroups, float max_grad_norm, float eps,
                           float* clip_out, void* workspace, size_t workspace_bytes, void* stream);

/* ---- caller glue: filter, depth sort, gather, activations ---------------------- */
/*
 * Pre-activation Gaussian parameters as the model stores them (model.py:138-169):
 * means N x 3, pre_quats N x 4, pre_scales N x 3 (log scales), colours N x C,
 * pre_phase N x C, pre_opac N, pre_planes N x K (plane logits); float32, device.
 */
typedef struct {
  int N, K, C;
  const float* means;
  const float* pre_quats;
  const float* pre_scales;
  const float* colours;
  const float* pre_phase;
  const float* pre_opac;
  const float* pre_planes;
} cvhrf_gaussians;

/*
 * Scene.render up to the splat call (model.py:1365-1402 with apply_activations
 * :595-608 and the straight-through one-hot :41-56), fused: X_cam = X R + T (R 3x3
 * row-major, T 3; device), depth sort of the rows with near < z < far (rows outside
 * sort last and keep their out-of-range depth, so the rasterizer culls them), gather
 * and activation.  Outputs are the N rows in that order (the rasterizer's inputs);
 * order[s] is the parameter row of sorted row s.  No host synchronisation.
 */
size_t cvhrf_scene_workspace_bytes(int N);
int cvhrf_scene_prepare(const cvhrf_gaussians* gaussians, const float* R, const float* T, float near_plane,
                        float far_plane, void* workspace, size_t workspace_bytes, int32_t* order,
                        float* cam_means, float* z_vals, float* quats, float* scales, float* colours,
                        float* phase, float* opacities, float* plane_probs, void* stream);
/*
 * cvhrf_scene_prepare restricted to a set of planes (bit p of owned_planes = plane p,
 * K <= 32; 0xFFFFFFFF = all): rows whose one-hot plane is not owned are sorted last and
 * culled like rows outside (near, far).  Used by plane-parallel training, where each GPU
 * renders only the planes it owns.  No counterpart in the reference.
 */
int cvhrf_scene_prepare_owned(const cvhrf_gaussians* gaussians, const float* R, const float* T, float near_plane,
                              float far_plane, uint32_t owned_planes, void* workspace, size_t workspace_bytes,
                              int32_t* order, float* cam_means, float* z_vals, float* quats, float* scales,
                              float* colours, float* phase, float* opacities, float* plane_probs, void* stream);
/* Backward of cvhrf_scene_prepare: gradients of the sorted rows -> parameter rows (every row written). */
int cvhrf_scene_backward(const cvhrf_gaussians* gaussians, const float* R, const int32_t* order,
                         const float* g_cam_means, const float* g_quats, const float* g_scales,
                         const float* g_colours, const float* g_phase, const float* g_opacities,
                         const float* g_plane_probs, float* d_means, float* d_pre_quats, float* d_pre_scales,
                         float* d_colours, float* d_pre_phase, float* d_pre_opacities, float* d_pre_planes,
                         void* stream);

/* ---- binning primitives ----------------------------------------------------- */
/*
 * The scan and the stable radix sort the rasterizer's binning uses, as standalone calls
 * (replace cub::DeviceScan::InclusiveSum, rasterizer_splat.cu:427, and
 * cub::DeviceRadixSort::SortPairs, :475-480).  Both are single-pass with decoupled
 * look-back: one launch per scan, one histogram launch plus one launch per 8-bit pass
 * per sort.  The sort orders (keys, values) in place by key bits [begin_bit, end_bit),
 * stably; n < 2^30.
 * cvhrf_lookback_timeouts: how many look-back waits ran out of their iteration limit
 * since the library was loaded (each invalidates that result; expected 0; synchronises).
 */
size_t cvhrf_sort_pairs_workspace_bytes(int n);
int cvhrf_sort_pairs_u32(uint32_t* keys, uint32_t* values, int n, int begin_bit, int end_bit,
                         void* workspace, size_t workspace_bytes, void* stream);
size_t cvhrf_inclusive_scan_workspace_bytes(int n);
int cvhrf_inclusive_scan_u32(const uint32_t* in, uint32_t* out, int n, void* workspace,
                             size_t workspace_bytes, void* stream);
int cvhrf_lookback_timeouts(void);
/*
 * How many waits of the propagation column passes on their bulk (TMA) column copies ran
 * out of their iteration limit since the library was loaded (each invalidates that call's
 * result; expected 0; synchronises).
 */
int cvhrf_copy_wait_timeouts(void);

/* ---- L2 intensity loss of the training iteration --------------------------- */
/*
 * loss = mean_i ((|holo_i|^2 - target_i)^2) over n complex64 holo values and n float
 * targets (train.py computes this with torch elementwise ops).  One launch; *loss is
 * a DEVICE float.  The workspace (cvhrf_intensity_loss_workspace_bytes) holds block
 * partials and a completion counter: zero it once with
 * cvhrf_intensity_loss_init_workspace; each call leaves it ready for the next (also
 * when replayed from a captured graph).  Calls sharing a workspace must be ordered on
 * one stream.  holo must be 16-byte and target 8-byte aligned.  The partial sums are
 * combined in a fixed order, so the result is deterministic.
 * Backward: grad_holo = (*grad_loss / n) * 2 r * 2 holo, r = |holo|^2 - target, with
 * *grad_loss a DEVICE float (the upstream gradient).
 */
size_t cvhrf_intensity_loss_workspace_bytes(int n);
int cvhrf_intensity_loss_init_workspace(void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_intensity_loss(const void* holo, const float* target, int n, float* loss,
                         void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_intensity_loss_backward(const void* holo, const float* target, int n, const float* grad_loss,
                                  void* grad_holo, void* stream);


/* ---- adaptive density control and opacity regularisation ------------------- */
/*
 * Gaussians.density_control (model.py:626-1047) on the device.  A Gaussian set is the
 * seven parameter arrays of cvhrf_gaussians plus their gradients (same shapes;
 * grad_pre_opac and grad_pre_planes may be null, read as zeros, as the reference does
 * when those .grad are None).  With g = |grad_means_i|, a = mean_j exp(pre_scales_ij),
 * o = sigmoid(pre_opac_i):
 *   keep  = o >= opacity_threshold
 *   clone = keep & g >= grad_threshold & a < small_scale_threshold
 *   split = keep & g >= grad_threshold & a > large_scale_threshold
 * Output rows, in this order: every kept row (unchanged, with its gradient); one clone
 * per cloned row (means + clone_offset_factor * grad / max(|grad|, 1e-8), opacity
 * logit(1 - sqrt(1 - o)) as log(c / (1 - c + 1e-6) + 1e-6), gradient copied); then the
 * first and then the second child of every split row (pre_scales - log(split_factor),
 * means +/- R(q / |q|) (noise_r * 0.5 * a), gradients halved).  noise is n_split x 3
 * standard-normal draws (row r for the r-th split row in row order), the draws the
 * reference takes with torch.randn_like(means_split).
 *
 * cvhrf_density_classify writes counts[0..3] (DEVICE u32) = kept, cloned, split and
 * pruned rows; the output holds counts[0] + counts[1] + 2 counts[2] rows.  The workspace
 * (cvhrf_density_workspace_bytes(N)) carries the row classification to
 * cvhrf_density_apply, which writes the output set (out->N = that row count, out->K, C
 * as in; its gradient pointers must all be non-null).  Output arrays must not overlap
 * the input ones.
 */
typedef struct {
  int N, K, C;
  float* means;
  float* pre_quats;
  float* pre_scales;
  float* colours;
  float* pre_phase;
  float* pre_opac;
  float* pre_planes;
  float* grad_means;
  float* grad_pre_quats;
  float* grad_pre_scales;
  float* grad_colours;
  float* grad_pre_phase;
  float* grad_pre_opac;
  float* grad_pre_planes;
} cvhrf_gaussian_set;

typedef struct {
  float grad_threshold, opacity_threshold, small_scale_threshold, large_scale_threshold;
  float split_factor, clone_offset_factor;
} cvhrf_density_params;

size_t cvhrf_density_workspace_bytes(int N);
int cvhrf_density_classify(const cvhrf_gaussian_set* in, const cvhrf_density_params* params, void* workspace,
                           size_t workspace_bytes, uint32_t* counts, void* stream);
int cvhrf_density_apply(const cvhrf_gaussian_set* in, const cvhrf_density_params* params, const float* noise,
                        const void* workspace, size_t workspace_bytes, const cvhrf_gaussian_set* out, void* stream);
/*
 * Gaussians.opacity_regularization (model.py:1049-1077), in place: with o =
 * sigmoid(pre_opac_i), pre_opac_i -= amount / max(o (1 - o), 1e-6); *affected (DEVICE
 * u32, overwritten) = the number of rows with o > amount.
 */
int cvhrf_opacity_regularization(float* pre_opac, int N, float amount, uint32_t* affected, void* stream);


/* ---- multiplane reconstruction loss ---------------------------------------- */
/*
 * The training loss over the K reconstructed planes (train.py:293-304 with
 * multiplane_loss_odak.__call__, utils/propagator.py:138-169), in one launch.
 * fields: K x C x S x S complex64 plane fields (the SLM -> plane propagation's output).
 * For each plane p, channel c and pixel of the centred H x W crop (odak crop_center:
 * rows S/2 - H/2 ..., H and W even as in the reference):
 *   x = clamp(s_c |f|^2, 0, 1),  s_c = channel_scale[c] (HOST, C <= 8; null = 1; the sum
 *       over frames of the channel's squared laser power, utils/propagator.py:612-634)
 *   loss = sum over planes of w0 mean((x - t)^2) + w1 mean((x m - t m)^2) + w2 mean((x t - t t)^2)
 * with targets t and masks m (K x C x H x W float, device), weights w (HOST, 3 floats),
 * means over C x H x W.  pred (K x C x H x W) receives x; *loss is a DEVICE float.
 * The workspace (cvhrf_multiplane_loss_workspace_bytes) is zeroed once with
 * cvhrf_multiplane_loss_init_workspace and left ready by every call (calls sharing it
 * must be ordered on one stream); the reduction order is fixed (deterministic).
 * Backward: grad_fields (K x C x S x S, every element written, zero outside the crop)
 * from *grad_loss (DEVICE float) and an optional extra gradient grad_pred with respect
 * to pred (K x C x H x W, e.g. from an SSIM term; null = none); clamp passes the
 * gradient where 0 <= s_c |f|^2 <= 1, as torch.clamp does.
 */
size_t cvhrf_multiplane_loss_workspace_bytes(void);
int cvhrf_multiplane_loss_init_workspace(void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_multiplane_loss(const void* fields, int K, int C, int S, int H, int W, const float* channel_scale,
                          const float* targets, const float* masks, const float* weights, float* pred, float* loss,
                          void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_multiplane_loss_backward(const void* fields, int K, int C, int S, int H, int W, const float* channel_scale,
                                   const float* targets, const float* masks, const float* weights,
                                   const float* grad_loss, const float* grad_pred, void* grad_fields, void* stream);


/* ---- hologram -> SLM field of the training loss ------------------------------ */
/*
 * train.py:280-283 with the field formation of utils/propagator.py:612-620, fused: for
 * the C x n complex64 hologram h (channel-major),
 *   phi = angle(h) mod 2 pi, m = mean of phi over all C n values, field[c] = |h| exp(i (phi - m) s_c)
 * with s_c = phase_scale[c] (HOST, C <= 8; null = 1).  *mean (DEVICE float) receives m and
 * is passed back to the backward, which writes grad_holo (torch's complex-gradient
 * convention; zero where h = 0) from grad_field.  The workspace
 * (cvhrf_hologram_field_workspace_bytes) is zeroed once with
 * cvhrf_hologram_field_init_workspace and left ready by every call.  The forward and the
 * backward use the same completion counter and partial sums in it, so every call sharing
 * one workspace (forward or backward, eager or inside a graph) must be ordered on one
 * stream; concurrent users (two streams, two graphs replaying at once) each need their
 * own workspace.  Reductions are in a fixed order (deterministic).
 */
size_t cvhrf_hologram_field_workspace_bytes(void);
int cvhrf_hologram_field_init_workspace(void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_hologram_field(const void* holo, int C, long long n, const float* phase_scale, void* field, float* mean,
                         void* workspace, size_t workspace_bytes, void* stream);
int cvhrf_hologram_field_backward(const void* holo, int C, long long n, const float* phase_scale, const float* mean,
                                  const void* grad_field, void* grad_holo, void* workspace, size_t workspace_bytes,
                                  void* stream);

#ifdef __cplusplus
}
#endif
#endif /* CVHRF_H_ */

/*
 * muon_polar_sm100.h -- C ABI of the B200 (sm_100a) Polar Express step.
 *
 * One Polar Express (Newton-Schulz) step of Muon:
 *     A = X . X^T            (kernel 1, symmetric Gram, bf16 storage)
 *     P = b . A + c . A . A  (kernel 2, polynomial, bf16 storage)
 *     Y = a . X + P . X      (kernel 3, apply)
 * for a batch of bf16 matrices X[batch][m][n] (row stride ldx elements,
 * batch stride m*ldx elements).
 *
 * Every entry point
 *   - takes plain device pointers, sizes and a cudaStream_t passed as void*,
 *   - allocates nothing (the caller owns every buffer),
 *   - launches asynchronously on `stream` and returns a status code:
 *       0                      success
 *       < 0                    MUON_POLAR_ERR_* (argument / setup error,
 *                              nothing was launched)
 *       > 0                    the cudaError_t reported by the launch.
 *
 * The reference (Ascend 950PR build) exposes three launchers with the
 * signature `void launch_xxx(void* in..., void* out, void* tilingDevice,
 * uint32_t blockDim, aclrtStream stream)`:
 *   csrc/muon_polar_unified_ascend950.asc:512-517   launch_muon_gram_lowlevel_fused
 *   csrc/muon_polar_unified_ascend950.asc:1030-1035 launch_muon_cube2_p_fused
 *   csrc/muon_polar_unified_ascend950.asc:1535-1540 launch_muon_cube3_fused_lowlevel
 * declared at csrc/muon_polar_step_binding.cpp:65-70.  Here the tiling
 * struct and block count are computed inside the library (they depend only
 * on sizes and the device), so each launcher takes sizes instead.
 */
#ifndef MUON_POLAR_SM100_H
#define MUON_POLAR_SM100_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MUON_POLAR_ABI_VERSION 1

#define MUON_POLAR_OK 0
#define MUON_POLAR_ERR_INVALID_ARGUMENT (-1)
#define MUON_POLAR_ERR_UNSUPPORTED_DEVICE (-2)
#define MUON_POLAR_ERR_ALIGNMENT (-3)
#define MUON_POLAR_ERR_TENSOR_MAP (-4)
#define MUON_POLAR_ERR_WORKSPACE (-5)
#define MUON_POLAR_ERR_DRIVER (-6)
#define MUON_POLAR_ERR_STATIC_SCRATCH (-7)

/* Size of the split-K scratch array built into the library for
 * muon_polar_gram_static_scratch_sm100: 1 KiB of counters + 80 partial bands
 * of 256 KiB (20 MiB + 1 KiB per GPU that loads the library). */
#define MUON_POLAR_STATIC_SCRATCH_BYTES ((size_t)1024 + (size_t)80 * (size_t)262144)

/* Bits of the device watchdog word (muon_polar_read_device_status). A bit is
 * set when a bounded wait inside a kernel gave up; the kernel then left its
 * loop, drained what it had in flight, released its tensor memory and
 * returned instead of hanging. */
#define MUON_POLAR_WATCHDOG_PRODUCER 0x1u
#define MUON_POLAR_WATCHDOG_MMA 0x2u
#define MUON_POLAR_WATCHDOG_EPILOGUE 0x4u
#define MUON_POLAR_WATCHDOG_DRAIN 0x8u
#define MUON_POLAR_WATCHDOG_DEPENDENCY 0x10u

/* Library version of this ABI (MUON_POLAR_ABI_VERSION). */
int muon_polar_abi_version(void);

/* Human-readable text for a status code returned by any entry point. */
const char* muon_polar_status_string(int status);

/* Rows of the square Gram/polynomial buffers for `m` rows of X: m rounded up
 * to 256, the height of a CTA-pair tile (the reference rounds to 128,
 * csrc/muon_polar_step_binding.cpp:630; the extra rows are zeros and do not
 * change any result). */
int64_t muon_polar_padded_rows(int64_t m);

/* Bytes of the workspace muon_polar_step_sm100 needs: A and P, each
 * [batch][Mp][Mp] bf16 with Mp = muon_polar_padded_rows(m).  Replaces the two
 * at::empty calls of csrc/muon_polar_step_binding.cpp:646,657. */
size_t muon_polar_workspace_bytes(int64_t batch, int64_t m);

/* Scratch.  Its first 1024 bytes are counters that must be zero before the
 * first call (muon_polar_scratch_init) and that every call leaves at zero:
 * the fused step keeps its per-matrix dependency counts there, split-K its
 * arrival counts.  muon_polar_scratch_bytes() is at least 1024.
 *
 * Split-K.  When a problem has fewer 256 x 256 output tiles than
 * the device has SM pairs (small M), kernels 1 and 2 cut each tile's K range
 * into up to 4 work items and reduce the fp32 partials -- always in the same
 * split order, so results are deterministic.  The reduction needs scratch
 * memory after the counters: muon_polar_scratch_bytes() covers it on the
 * current device.  Calls that share one scratch buffer must be
 * ordered (same stream).  Passing scratch = NULL (or too few bytes) turns
 * split-K off; results then come from the unsplit K order. */
size_t muon_polar_scratch_bytes(int64_t batch, int64_t m, int64_t n);

/* Zeroes the counter area of a scratch buffer (cudaMemsetAsync on `stream`).
 * Needed once after allocation, and again after a watchdog report. */
int muon_polar_scratch_init(void* scratch, size_t scratch_bytes, void* stream);

/* Kernel (1): gram[b] = X[b] . X[b]^T, bf16 [batch][Mp][Mp] (row stride Mp).
 * fp32 accumulation, one round-to-nearest-even to bf16.  Only tiles with
 * tile_row <= tile_col are computed; each is written at (tm,tn) and mirrored
 * to (tn,tm).  Rows/cols >= m are written as zeros.
 * Requirements: x 16-byte aligned, ldx % 8 == 0, ldx >= n, gram 16-byte
 * aligned.  scratch: see muon_polar_scratch_bytes (may be NULL).
 * Replaces launch_muon_gram_lowlevel_fused (asc:512-517). */
int muon_polar_gram_sm100(const void* x, void* gram, int64_t batch, int64_t m,
                          int64_t n, int64_t ldx, void* scratch,
                          size_t scratch_bytes, void* stream);

/* Kernel (1) for callers that cannot allocate device memory.  It has no
 * counterpart in the reference.
 *
 * Some callers have no way to hand this library scratch memory: a plugin
 * or real-time host that works inside a fixed device-memory budget, code
 * running next to a framework whose allocator has already reserved nearly
 * all of the GPU (so a cudaMalloc of its own fails or fragments that pool),
 * or a hot path that must not call cudaMalloc/cudaFree because they can
 * synchronise the device.  For them this entry computes exactly what
 * muon_polar_gram_sm100 computes on its CTA-pair path with split-K -- same
 * tiles, same split plan, same reduction order, so the same bits -- but
 * takes its split-K scratch from an array compiled into the library
 * (MUON_POLAR_STATIC_SCRATCH_BYTES per GPU, held until the process exits).
 * The caller still passes x and gram; nothing is allocated.
 *
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress, with that device current); make that first call
 *    before starting any stream capture.  A lookup that fails is returned
 *    as its cudaError_t and is tried again by the next call; only a
 *    successful lookup is kept.
 *  - The array is shared by every call on a device and keeps the previous
 *    call's contents; each call clears the counter part itself
 *    (cudaMemsetAsync on `stream`).  Calls whose executions overlap on the
 *    GPU (different streams, not ordered) race on the array and produce
 *    wrong results: order them.
 *  - A problem whose split plan needs more than the array (or than the
 *    budget set by muon_polar_set_static_scratch_limit) returns
 *    MUON_POLAR_ERR_STATIC_SCRATCH and launches nothing.
 * Arguments and layout as for muon_polar_gram_sm100. */
int muon_polar_gram_static_scratch_sm100(const void* x, void* gram, int64_t batch,
                                         int64_t m, int64_t n, int64_t ldx,
                                         void* stream);

/* Kernel (1), fp32 output variant: partial Gram in fp32 for the column-sharded
 * multi-GPU path (the partials are summed across ranks before kernel 2).
 * Same layout and requirements as muon_polar_gram_sm100, gram is float. */
int muon_polar_gram_f32_sm100(const void* x, void* gram_f32, int64_t batch,
                              int64_t m, int64_t n, int64_t ldx, void* scratch,
                              size_t scratch_bytes, void* stream);

/* Kernel (1), fp32 output, on a band of rows: the upper tiles of rows
 * [row_begin, row_begin + row_count) of gram_f32 (both multiples of 256,
 * inside muon_polar_padded_rows(m)), each stored with its mirror.  Run for
 * consecutive bands from row 0 on, the rows of a band are complete (both
 * triangles) as soon as its call has run, so a column-sharded caller can
 * all-reduce band i while band i + 1 computes; after the last band the
 * buffer equals muon_polar_gram_f32_sm100's.  `sm_reserve` SMs are left
 * free (rounded up to whole clusters of two) for kernels on other streams,
 * such as the collective.  No counterpart in the reference (single device). */
int muon_polar_gram_f32_band_sm100(const void* x, void* gram_f32, int64_t batch, int64_t m,
                                   int64_t n, int64_t ldx, int64_t row_begin, int64_t row_count,
                                   int sm_reserve, void* scratch, size_t scratch_bytes,
                                   void* stream);

/* Packed upper triangle, for column-sharded multi-GPU callers (no
 * counterpart in the reference, which runs on one device).  A symmetric
 * Mp x Mp matrix is cut into 256 x 256 units; the d (d + 1) / 2 units (I, J)
 * with I <= J (d = Mp / 256) are stored one after another, row by row of the
 * unit grid, each as a dense row-major 256 x 256 block: [batch][units][256][256].
 * The lower-left 128 x 128 quarter of a diagonal unit (I, I) is unspecified
 * (it mirrors the upper-right one).  A collective on the packed form moves
 * (d + 1) / (2 d) of the bytes of the full matrix.
 *
 * muon_polar_packed_units: units per matrix for `m` rows of X.
 * muon_polar_gram_f32_packed_sm100: kernel (1), fp32, written packed (no
 *   mirror), e.g. a rank's partial Gram before a reduce-scatter of the units.
 *   Arguments as for muon_polar_gram_f32_sm100.
 * muon_polar_poly_packed_sm100: kernel (2) on units [unit_begin, unit_begin +
 *   unit_count) of each matrix, read from the full bf16 gram [batch][Mp][Mp],
 *   written into their places in the packed bf16 buffer (other units are not
 *   touched); the arithmetic of muon_polar_poly_sm100.
 * muon_polar_unpack_sym_sm100: packed bf16 units -> the full symmetric
 *   [batch][Mp][Mp] bf16 matrix (each unit and, off the diagonal, its
 *   transpose). */
int64_t muon_polar_packed_units(int64_t m);
int muon_polar_gram_f32_packed_sm100(const void* x, void* packed_f32, int64_t batch, int64_t m,
                                     int64_t n, int64_t ldx, void* scratch, size_t scratch_bytes,
                                     void* stream);
int muon_polar_poly_packed_sm100(const void* gram, void* packed_poly, int64_t batch, int64_t mp,
                                 int64_t unit_begin, int64_t unit_count, float b, float c,
                                 void* stream);
int muon_polar_unpack_sym_sm100(const void* packed, void* full, int64_t batch, int64_t mp,
                                void* stream);

/* Kernel (2): poly[b] = bf16( b*f32(gram[b]) + c*(gram[b].gram[b])_f32 ),
 * both [batch][Mp][Mp] bf16, Mp a multiple of 128 (256 for the CTA-pair
 * kernels; muon_polar_padded_rows gives 256-multiples).  Products and the
 * sum are separately rounded fp32 operations (no FMA), as in
 * csrc/muon_polar_unified_ascend950.asc:929-940.  Upper tiles are computed
 * and mirrored.  Replaces launch_muon_cube2_p_fused (asc:1030-1035). */
int muon_polar_poly_sm100(const void* gram, void* poly, int64_t batch,
                          int64_t mp, float b, float c, void* scratch,
                          size_t scratch_bytes, void* stream);

/* Kernel (2) on a slab of rows: rows [row_begin, row_begin + row_count) of
 * poly[b], written in place into the full [batch][Mp][Mp] bf16 buffer `poly`
 * (whole rows: both triangles, no mirror), with the arithmetic of
 * muon_polar_poly_sm100.  Mp, row_begin and row_count are multiples of 256.
 * For multi-GPU callers that split kernel (2) by row slabs and then gather
 * the slabs (the reference runs kernel 2 on one device only). */
int muon_polar_poly_rows_sm100(const void* gram, void* poly, int64_t batch,
                               int64_t mp, int64_t row_begin, int64_t row_count,
                               float b, float c, void* stream);

/* Kernel (3): y[b] = bf16(T) + bf16(alpha_bf16 * x) with T = (poly[b].x[b])
 * accumulated in fp32 and the final add done on bf16 values, as in
 * csrc/muon_polar_unified_ascend950.asc:1472-1476; alpha_bf16 is `a`
 * rounded to bf16 (csrc/muon_polar_step_binding.cpp:156-162).  poly is
 * [batch][Mp][Mp] bf16; x and y are [batch][m][ld] with ldx, ldy % 8 == 0.
 * Replaces launch_muon_cube3_fused_lowlevel (asc:1535-1540). */
int muon_polar_apply_sm100(const void* poly, const void* x, void* y,
                           int64_t batch, int64_t m, int64_t n, int64_t ldx,
                           int64_t ldy, float a, void* stream);

/* The whole step: kernels 1, 2, 3 back to back on `stream` (programmatic
 * dependent launch lets each kernel's prologue overlap the previous
 * kernel's tail).  workspace must hold muon_polar_workspace_bytes(batch, m)
 * bytes, 16-byte aligned; scratch as for kernels 1 and 2 (may be NULL).
 * y must not alias x.
 * Replaces the launch sequence of csrc/muon_polar_step_binding.cpp:644-666. */
int muon_polar_step_sm100(const void* x, void* y, void* workspace,
                          size_t workspace_bytes, void* scratch,
                          size_t scratch_bytes, int64_t batch, int64_t m,
                          int64_t n, int64_t ldx, int64_t ldy, float a,
                          float b, float c, void* stream);

/* M > N without transposed copies.  The reference's Python wrapper runs a
 * tall X (M > N) as polar_step(X^T).mT, making two transposed copies
 * (muon_ascend950/ops.py:27-32).  These entries compute the same result in
 * X's own layout:
 *     A = X^T . X          [batch][Np][Np] bf16, Np = muon_polar_padded_rows(n)
 *     P = b . A + c . A . A
 *     Y = a . X + X . P    (= (a . X^T + P . X^T)^T, P symmetric)
 * with the arithmetic of kernels 1-3 (fp32 accumulation, the same epilogue
 * roundings).  The Gram reads X with M-contiguous ("MN-major") tiles.
 * x and y are [batch][m][ld] with ldx, ldy % 8 == 0, any m and n.
 *
 * muon_polar_gram_t_sm100: kernel (1) on X^T; rows/cols >= n of gram are
 *   zeros.  scratch as for kernel (1); muon_polar_scratch_bytes(batch, n, m)
 *   covers it.
 * muon_polar_apply_t_sm100: kernel (3) on X^T; poly is [batch][Np][Np].
 *   Columns [n, align(n, 8)) of y (inside the row stride) may be written
 *   with zeros; later columns are not touched.
 * muon_polar_step_t_sm100: the three kernels; workspace must hold
 *   muon_polar_workspace_bytes(batch, n) bytes; y must not alias x. */
int muon_polar_gram_t_sm100(const void* x, void* gram, int64_t batch, int64_t m,
                            int64_t n, int64_t ldx, void* scratch, size_t scratch_bytes,
                            void* stream);
int muon_polar_apply_t_sm100(const void* poly, const void* x, void* y, int64_t batch,
                             int64_t m, int64_t n, int64_t ldx, int64_t ldy, float a,
                             void* stream);
int muon_polar_step_t_sm100(const void* x, void* y, void* workspace, size_t workspace_bytes,
                            void* scratch, size_t scratch_bytes, int64_t batch, int64_t m,
                            int64_t n, int64_t ldx, int64_t ldy, float a, float b, float c,
                            void* stream);

/* `steps` Polar Express steps (the reference's caller loop,
 * examples/five_steps.py:18-21, over polar_step) with coefficient rows
 * coefficients[3*i .. 3*i+2] = (a, b, c) (a host array).  Step 0 reads x
 * (row stride ldx); step i > 0 reads the previous step's output, kept in
 * buf0 / buf1 ([batch][m][ldb] bf16, ldb % 8 == 0; step i writes
 * buf[i % 2], the last step y).  buf0 may not be x, and y may not be the
 * last step's input (buf[(steps - 2) % 2]); buf0/buf1 may be NULL when
 * steps == 1.  workspace: muon_polar_workspace_bytes(batch, min(m, n)).
 * With m <= n and the step mode (muon_polar_set_step_mode) choosing the
 * fused kernel, up to 8 steps run as ONE persistent launch (per-matrix
 * dependencies across steps in the scratch counter area: the next step's
 * Gram of a matrix starts once the previous step's apply of that matrix is
 * complete); otherwise each step runs as muon_polar_step_sm100 (or its _t
 * form for m > n).  The result has the same bits either way when kernels
 * (1) and (2) do not split K. */
int muon_polar_steps_sm100(const void* x, void* y, void* buf0, void* buf1, int64_t ldb,
                           void* workspace, size_t workspace_bytes, void* scratch,
                           size_t scratch_bytes, int64_t batch, int64_t m, int64_t n,
                           int64_t ldx, int64_t ldy, const float* coefficients, int steps,
                           void* stream);

/* ------------------------------------------------------------------------
 * The caller side of the step, on the device (no counterpart in the
 * reference, which leaves the loop, the normalisation and the optimizer
 * update to its caller: README.md:5, examples/five_steps.py:18-21).
 *
 * muon_polar_express_sm100: `steps` Polar Express steps with coefficient rows
 * coefficients[3*i .. 3*i+2] = (a, b, c) (a host array), optionally after the
 * normalisation x / (||x||_F * 1.01 + 1e-6) of each matrix (fp32 norm, one
 * rounding to bf16).  x is [batch][m][ldx] (batch stride m*ldx), fp32
 * (x_dtype 0) or bf16 (x_dtype 1; without normalisation only bf16 with
 * ldx % 8 == 0, read in place by the first step).  y is [batch][m][ldy]
 * bf16 and must not alias x.  Tall x (m > n) runs the
 * transposed step.  workspace: muon_polar_express_workspace_bytes(batch, m,
 * n) bytes, 16-byte aligned; scratch as for muon_polar_step_sm100 (or its _t
 * form for tall x), sized by muon_polar_scratch_bytes(batch, min(m,n),
 * max(m,n)).  All launches are asynchronous on `stream`.
 *
 * muon_polar_update_sm100: one Muon update of a batch of parameter matrices
 *   buf <- lerp(buf, grad, 1 - momentum)            (momentum buffer, in place)
 *   v    = nesterov ? lerp(grad, buf, momentum) : buf
 *   X    = bf16( v / (||v||_F * 1.01 + 1e-6) )
 *   Y    = `steps` Polar Express steps of X
 *   p   <- round( p * (1 - lr * weight_decay) - lr * scale * Y )
 * param, grad and momentum are contiguous [batch][m][n] of one dtype: fp32
 * (dtype 0) or bf16 (dtype 1), pairwise distinct, 16-byte aligned.  The
 * arithmetic is fp32 with one rounding per stored value (lerp as torch.lerp
 * computes it).  workspace and scratch as for muon_polar_express_sm100. */
size_t muon_polar_express_workspace_bytes(int64_t batch, int64_t m, int64_t n);
int muon_polar_express_sm100(const void* x, int x_dtype, int64_t ldx, void* y, int64_t ldy,
                             void* workspace, size_t workspace_bytes, void* scratch,
                             size_t scratch_bytes, int64_t batch, int64_t m, int64_t n,
                             const float* coefficients, int steps, int normalize, void* stream);
int muon_polar_update_sm100(void* param, const void* grad, void* momentum, int dtype, void* workspace,
                      size_t workspace_bytes, void* scratch, size_t scratch_bytes, int64_t batch,
                      int64_t m, int64_t n, float lr, float momentum_coef, int nesterov,
                      float weight_decay, float scale, const float* coefficients, int steps,
                      void* stream);
/* Kernels launched by the two entries above (their elementwise stages; the
 * Polar Express kernels count in muon_polar_launch_count). */
uint64_t muon_polar_update_launch_count(void);

/* dst[i] = bf16_rne(src[i]) for i < count (fp32 Gram after the cross-rank
 * sum -> bf16 input of kernel 2). No counterpart in the reference, which has
 * no multi-device path. */
int muon_polar_cast_f32_bf16_sm100(const void* src, void* dst, int64_t count,
                                   void* stream);

/* Reads (and, if clear != 0, resets) the watchdog word of `device`.  This
 * call synchronises the device.  No counterpart in the reference, whose
 * kernels have no bounded waits (CheckAcl at binding.cpp:72-75 is the only
 * error path). */
int muon_polar_read_device_status(int device, uint32_t* flags, int clear);

/* Kernel selection, process-wide; returns the previous policy (or
 * MUON_POLAR_ERR_INVALID_ARGUMENT).
 *   0  by size (default): of 256 x 256 tiles on tcgen05 CTA pairs and
 *      128 x 128 tiles on single CTAs, the engine with the smaller estimated
 *      time (rounds of tiles over the device times the measured cost of the
 *      K loop of a tile);
 *   1  always CTA pairs;
 *   2  always single-CTA tiles.
 * The initial value comes from MUON_POLAR_PAIR (1 -> policy 1, 0 -> policy
 * 2).  Every policy computes the same mathematical result; the fp32
 * accumulation order (and so the last bit) may differ between them. */
int muon_polar_set_kernel_policy(int policy);

/* How muon_polar_step_sm100 runs a step, process-wide; returns the previous
 * mode (or MUON_POLAR_ERR_INVALID_ARGUMENT).
 *   0  by size (default): one fused launch for many small matrices (more
 *      256 x 128 Gram regions than CTA pairs, at most three times as many,
 *      and muon_polar_padded_rows(m) <= 768), where it measured 4-21% faster
 *      on B200; else three kernels;
 *   1  one fused persistent launch for all three stages, with per-matrix
 *      dependencies tracked in the scratch counter area (needs scratch);
 *   2  always three kernels.
 * Initial value from MUON_POLAR_FUSED (1 -> 1, 0 -> 2).  Results are the
 * same in every mode; the bits are identical when kernels (1) and (2) do not
 * split K (the fused launch never does; see muon_polar_set_split_mode). */
int muon_polar_set_step_mode(int mode);

/* Split-K of kernels (1) and (2) when scratch is given, process-wide;
 * returns the previous mode (or MUON_POLAR_ERR_INVALID_ARGUMENT).
 *   0  by size (default): only when the shorter K loops save more time than
 *      the partial sums' round trip through L2 costs;
 *   1  whenever the device has room for more work items than tiles;
 *   2  never.
 * Results are the same mathematical quantity in every mode; the fp32
 * summation order, and so the last bit, depends on the split. */
int muon_polar_set_split_mode(int mode);

/* Column halves of the single-CTA Gram and polynomial launches: when every
 * item fits on the device at once and no split-K is planned, off-diagonal
 * 128 x 128 tiles run as two 128 x 64 halves (twice the CTAs for the same
 * work; each half stores its columns and their mirror).  Returns the
 * previous mode:
 *   0  by size (default): whenever the halves fit in one round;
 *   1  the same (kept for symmetry with the other mode setters);
 *   2  never.
 * The results are bit-identical in every mode. */
int muon_polar_set_halves_mode(int mode);

/* K depth of the single-CTA bf16 Gram's pipeline stages (kernel 1 on small
 * problems).  Returns the previous mode:
 *   0  by size (default): three 64-column swizzle atoms per stage (K = 192,
 *      two stages in flight) when that covers at most 4% more K than
 *      two-atom stages (K = 128, three in flight) and the split-K planner,
 *      counting K in the deeper stages, plans no split;
 *   1  three atoms whenever that planner plans no split;
 *   2  never.
 * Unsplit, the results are bit-identical in every mode (the extra K reads
 * zeros); where a deep unsplit launch replaces a split-K plan, the last bits
 * differ as between split and unsplit results (the fp32 summation order). */
int muon_polar_set_stage_mode(int mode);

/* Number of 2-CTA clusters (tcgen05 CTA pairs) of the Gram kernel the
 * current device runs at once; the persistent grids are this many pairs. */
int muon_polar_device_pairs(int* pairs);

/* Number of kernels the library has launched in this process (all entry
 * points, all devices).  Used by benchmarks to report launch counts. */
uint64_t muon_polar_launch_count(void);

/* Number of tensor maps the library has encoded with the driver in this
 * process.  Maps are memoised on their arguments (address, sizes, strides,
 * box), so repeated calls on the same buffers encode nothing; the binding
 * keeps the reference's launch-state caches (binding.cpp:103-330) in this
 * form. */
uint64_t muon_polar_tensor_map_encodes(void);

/* Sets the limit of every bounded wait inside this library's kernels on the
 * current device (default 2 s): a wait that has not ended after `limit_ns`
 * nanoseconds of wall-clock time gives up, sets its watchdog bit
 * (muon_polar_read_device_status) and the kernel drains and returns.  The
 * previous limit is stored in *previous (may be NULL).  1000 <= limit_ns <=
 * 6e10.  Synchronous with respect to the host (cudaMemcpyToSymbol); call it
 * while no kernel of this library runs on the device.  No counterpart in the
 * reference, whose kernels have no bounded waits. */
int muon_polar_set_wait_limit_ns(uint64_t limit_ns, uint64_t* previous);

/* Budget of muon_polar_gram_static_scratch_sm100 in bytes of its built-in
 * array, process-wide: plans needing more are refused with
 * MUON_POLAR_ERR_STATIC_SCRATCH.  0 (or anything above the array's size)
 * means the whole array, the default.  Returns the previous budget. */
size_t muon_polar_set_static_scratch_limit(size_t bytes);

/* Host-side checks (no GPU needed), used by the test suite.
 *
 * muon_polar_decode_tile: the work-item enumeration the kernels use, run on
 *   the host: linear tile index -> out[0..2] = (batch, tile row, tile col).
 *   symmetric != 0: the upper-triangle tiles (tm <= tn) of tile rows
 *   first_row .. tiles_m - 1, row by row (tiles_per_batch of them; the
 *   reference enumerates the same set, asc:129-146 and 609-630); else the
 *   tiles_m x tiles_n grid in row-major order.
 * muon_polar_check_address_cache: exercises the per-device address cache of
 *   muon_polar_gram_static_scratch_sm100 with a stand-in lookup that fails
 *   once and then succeeds; returns 0 when a failure was reported and not
 *   kept, the retry succeeded and later calls reuse the cached address. */
int muon_polar_decode_tile(int64_t tile, int symmetric, int64_t tiles_m, int64_t tiles_n,
                           int64_t tiles_per_batch, int64_t first_row, int64_t* out);
int muon_polar_check_address_cache(void);

#ifdef __cplusplus
}
#endif

#endif /* MUON_POLAR_SM100_H */

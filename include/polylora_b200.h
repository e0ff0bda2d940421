/*
 * polylora_b200 — C ABI of the B200 (sm_100a) batched multi-adapter LoRA path.
 *
 * Every entry point takes plain device pointers, element counts and a CUDA
 * stream handle (cudaStream_t passed as void*), returns a PLORA_* status and
 * never throws across the boundary.  No entry point allocates device memory:
 * callers pass outputs and, where one is needed, a workspace sized by
 * plora_workspace_size().  Work is enqueued on `stream`; nothing synchronises
 * the host except plora_device_status().
 *
 * Layout conventions (all tensors contiguous, row-major):
 *   x        (num_rows, max_seq, in_features)      activation rows
 *   lora_a   (num_slots, in_features, max_rank)    per-slot LoRA A, rank-minor
 *   lora_b   (num_slots, max_rank, out_features)   per-slot LoRA B
 *   tmp      (num_rows, max_seq, max_rank)         shrink output / expand input
 *   y        (num_rows, max_seq, out_features)     base output, updated in place
 *   weight_indices (num_rows,) int64  slot of each row; slot 0 is "__base__"
 *   seq_lens       (num_rows,) int32  valid tokens of each row (right padded)
 *   lora_ranks     (num_slots,) int32 rank of each slot (0 = no-op)
 *   scalings       (num_slots,) fp32  alpha / rank of each slot
 * Token t = row * max_seq + m is active when m < min(seq_lens[row], max_seq)
 * and lora_ranks[weight_indices[row]] > 0.
 */
#ifndef POLYLORA_B200_H_
#define POLYLORA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define PLORA_DTYPE_F32 0
#define PLORA_DTYPE_F16 1
#define PLORA_DTYPE_BF16 2

/* status codes */
#define PLORA_OK 0
#define PLORA_ERR_INVALID_ARGUMENT 1 /* shapes, pointers or sizes rejected on the host */
#define PLORA_ERR_UNSUPPORTED 2      /* valid request this build does not handle     */
#define PLORA_ERR_CUDA 3             /* a CUDA runtime call failed                   */
#define PLORA_ERR_WORKSPACE 4        /* workspace missing or too small               */
#define PLORA_ERR_DEVICE 5           /* a kernel raised the device status word       */

/* device status bits (plora_device_status) */
#define PLORA_DEV_WAIT_TIMEOUT 1 /* a bounded pipeline wait expired; kernel returned early */
#define PLORA_DEV_SLOT_RANGE 2   /* a weight index outside [0, num_slots) was skipped      */
#define PLORA_DEV_RANK_RANGE 4   /* a rank outside [0, max_rank] was clamped               */
#define PLORA_DEV_IMAGE_RANGE 8  /* a slot-image record pointed outside the image: rank 0  */
#define PLORA_DEV_PADDING 16     /* an attention mask was not right-padded                */
#define PLORA_DEV_TOKEN_RANGE 32 /* a segment-table token id outside [0, num_tokens) skipped */

/* Library version string. */
const char* plora_version(void);

/* Human-readable text for a PLORA_* status code. */
const char* plora_status_string(int status);

/* Detail of the last failing call on this host thread ("" if none). */
const char* plora_last_error(void);

/* Reads (and with clear != 0, resets) the device status word of the current
 * device.  Synchronises the device.  No counterpart in the reference: the
 * reference's Triton kernels have no device-side error reporting. */
int plora_device_status(int32_t* status_out, int32_t clear);

/* Work-split threshold of the tensor-core shrink / expand, in tokens per SM:
 * calls whose num_tokens is at most this times the SM count spread each
 * slot's LoRA weights over the grid (the slot-grid kernels: one CTA per slot
 * and weight part, for batches of few tokens per adapter such as decode);
 * larger calls give each CTA a share of the tokens.  Default 16.  With
 * value >= 0 sets it (0: always the token split); returns the previous value.
 * Process-wide; results do not depend on it beyond fp32 summation order.
 * No counterpart in the reference. */
int64_t plora_weight_split_tokens_per_sm(int64_t value);

/* Kernel family of rank-16 calls of many tokens (max_rank 16, 16-bit types,
 * K % 512 == 0 and K <= 4096 for the shrink, N % 512 == 0 and N <= 4096 for
 * the expand).  2 (the default): they stream token rows through shared memory
 * by bulk copies and keep the slot's weights in registers, and
 * plora_sgmv_shrink_expand runs as one fused kernel in which each CTA expands
 * the share it has just shrunk (where the expand phase fits the shrink's
 * shared memory); 1: the same kernels, the combined call as two launches; 0:
 * the windowed tensor-core kernels that serve every other rank.  Values above
 * 2 mean 2; value < 0 only reads.  Returns the previous setting.
 * Process-wide.  The stream settings give bit-identical results; the windowed
 * kernels agree with them within the documented tolerance (fp32 summation
 * order).  No counterpart in the reference. */
int32_t plora_stream_kernels(int32_t value);

/* Sets the limit of every bounded pipeline wait on the current device to
 * limit_ns (default 1 s) and returns the previous one in *previous (if not
 * null).  A wait that runs out sets PLORA_DEV_WAIT_TIMEOUT, and the kernel
 * skips its remaining work and returns; with 0, any wait that is not complete
 * when first polled runs out.  Meant for tests of that path.  Synchronises
 * the device.  No counterpart in the reference. */
int plora_set_wait_limit_ns(uint64_t limit_ns, uint64_t* previous);

/* Workspace bytes needed by plora_build_segments, plora_sgmv_a_fwd and
 * plora_sgmv_b_fwd for a batch of num_rows x max_seq tokens over num_slots
 * slots (segment scratch plus, for the *_fwd calls, the table itself).
 * The workspace must be 256-byte aligned.  Returns 0 for arguments those
 * calls reject: negative sizes, num_rows x max_seq beyond INT32_MAX tokens,
 * num_slots outside [1, 4096]. */
size_t plora_workspace_size(int64_t num_rows, int64_t max_seq, int32_t num_slots);

/* ---------------------------------------------------------------------------
 * Segment table: rows grouped by slot, built on the device.
 * Replaces the host-synchronising schedule of the reference
 * (src/polylora/sgmv.py:29-61 _build_flat_schedule and the n_eff gather at
 * sgmv.py:304-309): the result stays on the device and needs no .item().
 *   slot_start  (num_slots + 1,) int32: exclusive prefix of active tokens per
 *               slot; slot_start[num_slots] is the active-token total.
 *   token_index (num_rows * max_seq,) int32: active token ids (row*max_seq+m)
 *               ordered by (slot, row, m); entries past the total are unused.
 * A token is active when its slot's rank in `lora_ranks` is > 0.
 * Batches of at most 1024 rows, 256 slots and 16384 tokens are built by one
 * kernel, larger ones by three; the table is the same either way, and the
 * workspace must be passed in both cases.
 * ------------------------------------------------------------------------- */
int plora_build_segments(const int64_t* weight_indices, const int32_t* seq_lens,
                         const int32_t* lora_ranks, int64_t num_rows, int64_t max_seq,
                         int32_t num_slots, int32_t* slot_start, int32_t* token_index,
                         void* workspace, size_t workspace_size, void* stream);

/* Checks on the stream that an attention mask is right-padded, without
 * reading anything back: mask is (rows, width), contiguous, elements of
 * mask_elem_bytes (1, 2, 4 or 8) bytes, treated as floats with mask_is_float
 * (2, 4 or 8 bytes; the sign bit is ignored); seq_lens[r] (int64) is row r's sum
 * as the caller computed it from the same mask.  A row that is not non-zero
 * exactly at positions < seq_lens[r] sets PLORA_DEV_PADDING in the device
 * status word, which plora_device_status() reports later.  Replaces the
 * host-synchronising comparison of src/polylora/context.py:37-45
 * (assert_right_padded) for callers that keep the forward free of host
 * synchronisation. */
int plora_check_right_padded(const void* mask, int32_t mask_elem_bytes, int32_t mask_is_float,
                             const int64_t* seq_lens, int64_t rows, int64_t width, void* stream);

/* Reference-compatible flat tile schedule: src/polylora/sgmv.py:29-61
 * (_build_flat_schedule).  cum_tiles (num_rows+1,) and num_n_tiles (num_rows,)
 * int32 are written on the device; the tile total is cum_tiles[num_rows]. */
int plora_flat_schedule(const int32_t* seq_lens, const int32_t* n_eff, int64_t num_rows,
                        int32_t block_m, int32_t block_n, int32_t* cum_tiles,
                        int32_t* num_n_tiles, void* stream);

/* ---------------------------------------------------------------------------
 * SGMV shrink (LoRA A, down-projection): src/polylora/sgmv.py:141-175
 * sgmv_lora_a_fwd(x, weights, seq_lens, weight_indices, lora_ranks, stack_num)
 *   tmp[t, n] = sum_k x[t, k] * lora_a[slot(t), k, n]  for n < min(rank*stack_num, max_rank)
 *   tmp[t, n] = 0 for the remaining n of an active token; inactive tokens are
 *   not written (the reference leaves them uninitialised).
 * Builds the segment table in `workspace`, then runs the shrink kernel.
 * ------------------------------------------------------------------------- */
int plora_sgmv_a_fwd(const void* x, const void* lora_a, void* tmp, const int32_t* seq_lens,
                     const int64_t* weight_indices, const int32_t* lora_ranks, int64_t num_rows,
                     int64_t max_seq, int64_t in_features, int64_t max_rank, int32_t num_slots,
                     int32_t stack_num, int32_t dtype, void* workspace, size_t workspace_size,
                     void* stream);

/* ---------------------------------------------------------------------------
 * SGMV expand (LoRA B, up-projection) with fused scaling and add-back:
 * src/polylora/sgmv.py:278-328
 * sgmv_lora_b_fwd(x, weights, seq_lens, weight_indices, lora_ranks, scalings, base_output)
 *   y[t, :] += scalings[slot] * sum_{k < min(rank, max_rank)} tmp[t, k] * lora_b[slot, k, :]
 * in place on y (the reference's base_output; callers pass zeros where the
 * reference would allocate them).  Rows of rank-0 slots and padding tokens are
 * left bit-identical.
 * ------------------------------------------------------------------------- */
int plora_sgmv_b_fwd(const void* tmp, const void* lora_b, void* y, const int32_t* seq_lens,
                     const int64_t* weight_indices, const int32_t* lora_ranks,
                     const float* scalings, int64_t num_rows, int64_t max_seq, int64_t max_rank,
                     int64_t out_features, int32_t num_slots, int32_t dtype, void* workspace,
                     size_t workspace_size, void* stream);

/* plora_sgmv_a_fwd without a caller-provided workspace, for callers that
 * cannot allocate device memory at call time: code running inside a region
 * that forbids cudaMalloc (it synchronises the device), embedders whose
 * memory is a fixed pool they do not control, and foreign-language callers
 * that own no CUDA allocator.  No counterpart in the reference (its operators
 * always allocate through torch).
 * Its scratch is a static device array of PLORA_NOALLOC_SCRATCH_BYTES that
 * every GPU loading this library holds until process exit; a batch whose
 * segment scratch + table (plora_workspace_size) exceeds it is rejected with
 * PLORA_ERR_UNSUPPORTED.  The first call on each device looks up the array's
 * device address (make that first call before any stream capture).  All
 * calls share the array: calls that overlap on the GPU (other streams,
 * other threads) race and must be serialised by the caller.  Nothing in the
 * array needs to start at zero; each call rewrites what it reads. */
#define PLORA_NOALLOC_SCRATCH_BYTES (8u << 20)
int plora_sgmv_a_fwd_noalloc(const void* x, const void* lora_a, void* tmp, const int32_t* seq_lens,
                             const int64_t* weight_indices, const int32_t* lora_ranks,
                             int64_t num_rows, int64_t max_seq, int64_t in_features,
                             int64_t max_rank, int32_t num_slots, int32_t stack_num, int32_t dtype,
                             void* stream);

/* Shrink over a prebuilt segment table (plora_build_segments).  Same math as
 * plora_sgmv_a_fwd; `lora_ranks` may hold ranks of a different module than
 * the table was built with: tokens whose slot rank is 0 here are skipped. */
int plora_sgmv_shrink(const void* x, const void* lora_a, void* tmp, const int32_t* lora_ranks,
                      const int32_t* slot_start, const int32_t* token_index, int64_t num_tokens,
                      int64_t in_features, int64_t max_rank, int32_t num_slots, int32_t stack_num,
                      int32_t dtype, void* stream);

/* Expand over a prebuilt segment table.  Same math as plora_sgmv_b_fwd. */
int plora_sgmv_expand(const void* tmp, const void* lora_b, void* y, const int32_t* lora_ranks,
                      const float* scalings, const int32_t* slot_start, const int32_t* token_index,
                      int64_t num_tokens, int64_t max_rank, int64_t out_features,
                      int32_t num_slots, int32_t dtype, void* stream);

/* Shrink then expand of one wrapped Linear over a prebuilt segment table:
 * tmp = x A[slot] (stack_num 1), then y += scale tmp B[slot] in place.  The
 * same math as plora_sgmv_shrink followed by plora_sgmv_expand, and the
 * call a layer of the reference makes twice (layers.py:42-58, the
 * _SGMV_LORA_A_FWD / _SGMV_LORA_B_FWD pair).  Issued together, the expand is
 * launched to overlap the end of the shrink: it stages its tables, its LoRA-B
 * windows and its first rows of y while the shrink finishes, and reads tmp
 * only once the shrink has completed. */
int plora_sgmv_shrink_expand(const void* x, const void* lora_a, void* tmp, const void* lora_b,
                             void* y, const int32_t* lora_ranks, const float* scalings,
                             const int32_t* slot_start, const int32_t* token_index,
                             int64_t num_tokens, int64_t in_features, int64_t max_rank,
                             int64_t out_features, int32_t num_slots, int32_t dtype,
                             void* stream);

/* ---------------------------------------------------------------------------
 * Token rows between host memory and the device, for the tokens of a segment
 * table only.  No reference counterpart: the reference operators take device
 * tensors (src/polylora/sgmv.py:141-175, 278-328), so a caller holding host
 * buffers copies every row in and out.  The LoRA op reads x and the base
 * output only at the tokens the table lists and updates the base output in
 * place (the reference's expand adds into y, sgmv.py:278-328), so an in-place
 * host caller needs just those rows on the bus.
 *
 * plora_gather_token_rows copies row t (row_bytes bytes) of host_rows to row t
 * of device_rows, and plora_scatter_token_rows row t of device_rows to row t of
 * host_rows, for every token t in token_index[0 : slot_start[num_slots]].
 * The kernel itself reads or writes the host rows over PCIe, so host_rows must
 * be page-locked and mapped (cudaHostAlloc, or cudaHostRegister with
 * cudaHostRegisterMapped; both ends of its num_tokens * row_bytes bytes are
 * checked with cudaPointerGetAttributes, and pageable memory is refused with
 * PLORA_ERR_INVALID_ARGUMENT before any launch).  row_bytes: a positive
 * multiple of 16; both buffers 16-byte aligned.  The table is read on the
 * device after the preceding work in `stream`; a token id outside [0,
 * num_tokens) is skipped and sets PLORA_DEV_TOKEN_RANGE. */
int plora_gather_token_rows(const void* host_rows, void* device_rows, int64_t row_bytes, int64_t num_tokens,
                            const int32_t* slot_start, const int32_t* token_index, int32_t num_slots,
                            void* stream);
int plora_scatter_token_rows(const void* device_rows, void* host_rows, int64_t row_bytes, int64_t num_tokens,
                             const int32_t* slot_start, const int32_t* token_index, int32_t num_slots,
                             void* stream);

/* ---------------------------------------------------------------------------
 * GPU slot refill: src/polylora/cache.py:97-150 (_allocate_or_evict zeroing +
 * _load_adapter_into_slot copies).  One pinned host->device copy of a packed
 * adapter image into `staging`, then one kernel that writes every module's
 * slot (A and B zero-padded to max_rank, rank, scale; absent modules become
 * rank 0 / scale 0).  Enqueued on `stream` (callers use a side stream and
 * order it against compute with events).
 *   modules      device array of plora_slot_module (see below)
 *   host_image   pinned packed adapter image (layout below), image_bytes long
 *   staging      device buffer of at least image_bytes
 * Image layout: num_modules records of plora_slot_record, then the data
 * blocks they point at (byte offsets from the image start):
 *   A block (rank x in_features) row-major and B block (out_features x rank)
 *   row-major: the factors as PEFT stores them (lora_A.weight, lora_B.weight);
 *   the fill writes them transposed into the slot layouts.
 * A record of nonzero rank whose blocks are not inside [0, image_bytes), or
 * not aligned to the element size, is not read: that module is filled as
 * rank 0 and the device status gets PLORA_DEV_IMAGE_RANGE.
 * ------------------------------------------------------------------------- */
typedef struct plora_slot_module {
  void* lora_a;     /* (num_slots, in_features, max_rank) */
  void* lora_b;     /* (num_slots, max_rank, out_features) */
  int32_t* ranks;   /* (num_slots,) */
  float* scales;    /* (num_slots,) */
  int64_t in_features;
  int64_t out_features;
} plora_slot_module;

typedef struct plora_slot_record {
  int64_t a_offset; /* byte offset of the A block in the image */
  int64_t b_offset; /* byte offset of the B block in the image */
  int32_t rank;     /* 0 = module absent from this adapter */
  float scale;      /* alpha / rank */
} plora_slot_record;

int plora_slot_fill(const plora_slot_module* modules, int32_t num_modules, int32_t slot,
                    int32_t num_slots, int64_t max_rank, int32_t dtype, const void* host_image,
                    size_t image_bytes, void* staging, size_t staging_bytes, void* stream);

/* Host only: packs the LoRA factors of a PEFT adapter's safetensors file
 * (`path`) for `modules` into a slot image in plora_slot_fill's layout
 * (records, then A (rank x in) and B (out x rank) blocks, 256-byte aligned;
 * scale = lora_alpha / rank; absent modules rank 0).  A module's weight is the
 * first key, in data-offset order (as safetensors' load_file returns them),
 * ending in "<module>.lora_A.<adapter_name>.weight"
 * or "<module>.lora_A.weight" (lora_B likewise), as in the reference's loader
 * (src/polylora/store.py).  Writes *image_bytes (also when the image is too
 * small: PLORA_ERR_WORKSPACE, nothing written) and dims[3 * i .. 3 * i + 2] =
 * rank, in_features, out_features of module i.  Handles the common case only:
 * PLORA_ERR_UNSUPPORTED when a LoRA tensor is missing, malformed, not of
 * `dtype`, of inconsistent rank, duplicated, or outside `modules`, and when
 * any tensor fails the safetensors format's own checks (known dtype, bytes
 * matching the shape, data blocks tiling the data section) or is empty (the
 * Python loader then takes the file and raises the reference's errors);
 * PLORA_ERR_INVALID_ARGUMENT when the file cannot be opened or read.  No
 * counterpart in the reference (its loader is Python). */
int plora_peft_pack(const char* path, const char* const* modules, int32_t num_modules,
                    const char* adapter_name, int32_t dtype, double lora_alpha, void* image,
                    size_t capacity, size_t* image_bytes, int64_t* dims);

#ifdef __cplusplus
}
#endif

#endif /* POLYLORA_B200_H_ */

/*
 * mentat_b200.h -- C ABI of libmentat_b200.so, the B200 (sm_100a) implementation of
 * MENTAT's entropy-gated prefix-tree decode path.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t, is
 * stream-ordered, never allocates, and returns an int status (MENTAT_OK == 0,
 * negative on argument or launch errors).  Errors that can only be known on
 * the device (out of blocks, refcount underflow, plan overflow) are written to
 * the cache's control words (ctrl[MENTAT_CTRL_ERROR], ctrl[MENTAT_CTRL_ERRARG])
 * and read by the host at its next synchronisation point.
 *
 * Reference interfaces each entry point replaces are cited as
 * <file>:<line> of SkyeGunasekaran/MENTAT.
 */
#ifndef MENTAT_B200_H
#define MENTAT_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MENTAT_ABI_VERSION 1

/* status codes (returned) and device error codes (ctrl[MENTAT_CTRL_ERROR]) */
#define MENTAT_OK 0
#define MENTAT_ERR_ARG (-1)          /* invalid argument */
#define MENTAT_ERR_CUDA (-2)         /* a launch failed */
#define MENTAT_ERR_UNSUPPORTED (-3)  /* shape / dtype not built */
#define MENTAT_DEV_OUT_OF_BLOCKS 1   /* paged_kv_cache.py:46-50 RuntimeError */
#define MENTAT_DEV_REF_FREE 2        /* paged_kv_cache.py:59 AssertionError */
#define MENTAT_DEV_RELEASE_FREE 3    /* paged_kv_cache.py:63 AssertionError */
#define MENTAT_DEV_PLAN_OVERFLOW 4   /* decode plan exceeded its workspace */
#define MENTAT_DEV_TABLE_OVERFLOW 5  /* a sequence outgrew max_blocks_per_seq */
#define MENTAT_DEV_DECODE_TIMEOUT 6  /* a bounded wait in a decode kernel gave up; that call's output is invalid */
#define MENTAT_DEV_BAD_BLOCK 7       /* a block table entry outside [0, num_blocks) (ctrl[ERRARG] = the entry),
                                        which the decode and gather kernels do not read; that call's output is
                                        invalid.  The reference asserts on bad block ids at paged_kv_cache.py:59,63 */

/* dtypes */
#define MENTAT_F32 0
#define MENTAT_BF16 1
#define MENTAT_F16 2

/* control words of the block allocator, int64 each */
#define MENTAT_CTRL_HEAD 0    /* free-ring pops so far (monotonic) */
#define MENTAT_CTRL_TAIL 1    /* free-ring pushes so far (monotonic); free = tail - head */
#define MENTAT_CTRL_PEAK 2    /* high-water mark of blocks in use (paged_kv_cache.py:41-43) */
#define MENTAT_CTRL_ERROR 3   /* first device error code, 0 if none */
#define MENTAT_CTRL_ERRARG 4  /* its argument (block id, slot) */
#define MENTAT_CTRL_ALLOCS 5  /* blocks allocated so far */
#define MENTAT_CTRL_COWS 6    /* copy-on-write block copies so far */
#define MENTAT_CTRL_WORDS 16

/*
 * Paged KV cache state, all device memory owned by the caller.
 * Replaces PagedKVCacheManager's pools, BlockAllocator and SequenceState
 * (core/paged_kv_cache.py:21-140).  Sequences live in slots [0, max_seqs).
 */
typedef struct mentat_kv_cache {
    int32_t num_layers;
    int32_t num_blocks;          /* max_blocks of the reference */
    int32_t block_size;
    int32_t num_kv_heads;
    int32_t head_dim;
    int32_t dtype;               /* MENTAT_F32 / MENTAT_BF16 / MENTAT_F16 */
    int32_t max_seqs;
    int32_t max_blocks_per_seq;
    void* k_pool;                /* [num_layers][num_blocks][block_size][num_kv_heads][head_dim] */
    void* v_pool;                /* same */
    int32_t* refcounts;          /* [num_blocks] */
    int32_t* free_ring;          /* [num_blocks], FIFO of free block ids */
    int64_t* ctrl;               /* [MENTAT_CTRL_WORDS] */
    int32_t* tables;             /* [num_layers][max_seqs][max_blocks_per_seq] */
    int32_t* nblocks;            /* [num_layers][max_seqs] table lengths */
    int32_t* ntok;               /* [num_layers][max_seqs] num_tokens */
    int32_t* tail;               /* [num_layers][max_seqs] tokens_in_last_block */
    int32_t* scratch;            /* [mentat_kv_scratch_ints(max_seqs)] */
} mentat_kv_cache;

int mentat_abi_version(void);
const char* mentat_status_string(int status);
int64_t mentat_kv_scratch_ints(int32_t max_seqs);

/* BlockAllocator.__init__ (paged_kv_cache.py:26-30): refcounts 0, every block
 * free, in the order given by initial_order (device int32[num_blocks]; NULL
 * means 0..num_blocks-1), which is also the pop order. */
int mentat_kv_init(const mentat_kv_cache* c, const int32_t* initial_order, cudaStream_t s);

/* allocate_sequence (paged_kv_cache.py:143-150): empty tables in every layer. */
int mentat_kv_seq_reset(const mentat_kv_cache* c, int32_t slot, cudaStream_t s);

/* fork_sequence (paged_kv_cache.py:152-170): copy every layer's table and
 * counters of parent_slot to child_slot and ref() every block.
 * max_nblocks is the parent's longest table (a launch-size hint). */
int mentat_kv_fork(const mentat_kv_cache* c, int32_t parent_slot, int32_t child_slot,
                   int32_t max_nblocks, cudaStream_t s);

/* free_sequence (paged_kv_cache.py:172-176): release() every block, layer by
 * layer in table order; blocks reaching refcount 0 join the free FIFO in that
 * order. */
int mentat_kv_free(const mentat_kv_cache* c, int32_t slot, int32_t max_nblocks, cudaStream_t s);

/* append_tokens_batched (paged_kv_cache.py:227-284): one token for each of n
 * sequences (slots, device int32[n]) in layer `layer`: new block when the tail
 * is full or the table empty, copy-on-write of a shared tail, then the scatter
 * of k/v rows ([n][num_kv_heads][head_dim], token stride k_stride/v_stride in
 * elements).  n <= 1024 per call.  An entry whose slot is -1 is skipped (padding
 * of a batch to a fixed size, e.g. a captured CUDA graph's). */
int mentat_kv_append_batched(const mentat_kv_cache* c, int32_t layer, const int32_t* slots,
                             int32_t n, const void* k, int64_t k_stride, const void* v,
                             int64_t v_stride, cudaStream_t s);

/* append_tokens (paged_kv_cache.py:178-225): n tokens for one sequence. */
int mentat_kv_append(const mentat_kv_cache* c, int32_t layer, int32_t slot, int32_t n,
                     const void* k, int64_t k_stride, const void* v, int64_t v_stride,
                     cudaStream_t s);

/* trim_to_window (paged_kv_cache.py:370-417), every layer of one sequence. */
int mentat_kv_trim(const mentat_kv_cache* c, int32_t slot, int32_t window, cudaStream_t s);

/* build_packed_kv's gather (paged_kv_cache.py:347-359): materialise the packed
 * (sum_len, num_kv_heads, head_dim) K and V of n sequences; cu_seqlens is the
 * device int32[n+1] prefix sum of their lengths. */
int mentat_kv_gather(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n,
                     const int32_t* cu_seqlens, int64_t total_tokens, void* out_k, void* out_v,
                     cudaStream_t s);

/*
 * Tree-aware paged GQA decode attention.  Replaces build_packed_kv + attn_decode
 * (paged_kv_cache.py:289-368, attention_backend.py:192-228 -> flash_attn varlen
 * or _sdpa_decode :99-168).  Sequences are the slots of the batch, in batch
 * order; KV blocks shared by adjacent sequences of the batch (found from the
 * block tables) are read once for all of them.  n <= 1024 per call.
 *
 * q:   [n][num_q_heads][head_dim], token stride q_stride (elements), cache dtype.
 * out: same layout, out_stride.
 * scale: softmax scale (the reference uses 1/sqrt(head_dim)).
 * workspace: device memory of mentat_decode_workspace_bytes(...) bytes.
 */
int64_t mentat_decode_workspace_bytes(int32_t n, int32_t num_q_heads, int32_t head_dim,
                                      int32_t max_parts);
int32_t mentat_decode_max_parts(int32_t n, int32_t max_len, int32_t block_size);
int mentat_paged_decode(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n,
                        const void* q, int64_t q_stride, int32_t num_q_heads, void* out,
                        int64_t out_stride, float scale, void* workspace, int64_t workspace_bytes,
                        int32_t max_parts, cudaStream_t s);

/* The same decode for another layer of the same step, with the plan that an
 * earlier mentat_paged_decode call left in the workspace.  Replaces the per-layer
 * build_packed_kv + attn_decode of decode_batch (generator_utils.py:381-410) for
 * every layer after the first: forks copy all layers' tables and a decode step
 * appends to every layer, so all layers share one sharing structure, and the
 * partition of the batch into shared segments and units found for one layer
 * holds for the others.  The workspace must hold the plan of a call on the same
 * stream with the same slots, n, num_q_heads and max_parts, made after the
 * sequences last changed in every layer.  A workspace planned for another n,
 * max_parts, GQA group or routing runs no unit, zeroes the output and records
 * MENTAT_DEV_PLAN_OVERFLOW. */
int mentat_paged_decode_reuse_plan(const mentat_kv_cache* c, int32_t layer, const int32_t* slots,
                                   int32_t n, const void* q, int64_t q_stride, int32_t num_q_heads,
                                   void* out, int64_t out_stride, float scale, void* workspace,
                                   int64_t workspace_bytes, int32_t max_parts, cudaStream_t s);

/*
 * Causal prefill attention over the paged cache.  Replaces attn_prefill
 * (attention_backend.py:175-189 -> flash_attn_func(causal=True) or
 * _sdpa_prefill :43-96) for one sequence whose K/V the caller has already
 * appended: query i (i < n) sits at position pos0 + i of the sequence in
 * slot[0] (device int32[1]) and attends to its positions 0 .. pos0 + i.
 * pos0 = 0 is a whole-prompt prefill, pos0 > 0 a chunk of a longer one.
 * q / out: [n][num_q_heads][head_dim] as in mentat_paged_decode.
 * workspace: mentat_decode_workspace_bytes(n, num_q_heads, head_dim,
 * max_parts) bytes with max_parts >= mentat_prefill_max_parts(c, n, pos0,
 * num_q_heads), the partials a query can have (1 when every query group's
 * tokens fit one unit; 0 for invalid arguments).
 * bf16 / fp16 caches with block_size 16 run on the tensor cores (out 16-byte
 * aligned with out_stride a multiple of 8: single-partial rows are written by
 * the unit kernel itself); fp32 on FFMA.  A max_parts below what the plan needs
 * returns MENTAT_ERR_ARG and launches nothing.  Sliding windows are not
 * supported.
 */
int32_t mentat_prefill_max_parts(const mentat_kv_cache* c, int32_t n, int32_t pos0, int32_t num_q_heads);
int mentat_paged_prefill(const mentat_kv_cache* c, int32_t layer, const int32_t* slot, int32_t n,
                         int32_t pos0, const void* q, int64_t q_stride, int32_t num_q_heads, void* out,
                         int64_t out_stride, float scale, void* workspace, int64_t workspace_bytes,
                         int32_t max_parts, cudaStream_t s);

/* Decode for callers that cannot allocate device memory when they call.
 * No counterpart in the reference.  Some hosts cannot hand this library a
 * workspace: a program that binds the C ABI directly has no caching allocator,
 * and a cudaMalloc per call would synchronise the whole device; a serving
 * runtime may reserve all device memory up front and forbid new allocations
 * while it serves.  This variant of mentat_paged_decode takes the same
 * arguments minus the workspace and uses a fixed scratch array compiled into
 * the library instead (MENTAT_NOALLOC_SCRATCH_BYTES, held on every GPU that
 * loads the library until the process exits).  It never allocates.
 *  - A request whose workspace (mentat_decode_workspace_bytes(n, num_q_heads,
 *    head_dim, max_parts)) exceeds the limit returns MENTAT_ERR_SCRATCH_LIMIT
 *    and launches nothing.
 *  - The first call on a device looks up the array's device address with that
 *    device current; make that first call before any stream capture.
 *  - Every call on a device shares the one array, and each call overwrites it
 *    (the plan resets its own counters): calls that overlap on the GPU, e.g. on
 *    two streams, race and must be serialised by the caller. */
#define MENTAT_NOALLOC_SCRATCH_BYTES (16 * 1024 * 1024)
#define MENTAT_ERR_SCRATCH_LIMIT (-4)
int mentat_paged_decode_noalloc(const mentat_kv_cache* c, int32_t layer, const int32_t* slots, int32_t n,
                                const void* q, int64_t q_stride, int32_t num_q_heads, void* out,
                                int64_t out_stride, float scale, int32_t max_parts, cudaStream_t s);

/* Test hook for the bounded waits of the tensor-core decode kernels.  No
 * counterpart in the reference.  With cycles > 0, every CTA of those kernels
 * first waits, for at most `cycles` clock cycles, on a barrier that nothing
 * arrives on; the wait gives up before the CTA has issued any copy or MMA, the
 * CTA takes its timeout path, and the call reports MENTAT_DEV_DECODE_TIMEOUT
 * in the cache's control words with its output zeroed.  0 (the default) turns
 * the hook off.  Applies to the current device, synchronously. */
int mentat_decode_set_wait_probe(int64_t cycles);

/* Stage timing of mentat_paged_decode with CUDA events recorded on the launch
 * stream, for up to max_records launches (0 disables).  No counterpart in the
 * reference; used by the benchmark's roofline report.  collect waits for the
 * last recorded launch and returns, in stage_ms[5], the summed milliseconds of
 * the plan (with the table compare), the FFMA units, the wide and the narrow
 * tensor-core units and the merge, plus the number of launches, and restarts
 * the record. */
int mentat_profile_enable(int32_t max_records);
int mentat_profile_collect(double* stage_ms, int32_t* launches);

/* Number of kernels this library has launched since it was loaded (all entry
 * points, devices and streams).  No counterpart in the reference; the
 * benchmark reads it around its timed region. */
int64_t mentat_kernel_launch_count(void);

/*
 * Fused entropy gate over the full vocabulary, one leaf per row.  Replaces
 * compute_entropy (generator_utils.py:196-202), apply_repetition_penalty
 * (:205-230), adaptive_threshold (:247-253), and the arithmetic of
 * MentatGenerator._step_leaf / _do_branch / _do_extend / _soft_explore_factor
 * (generator.py:275-374).
 */
#define MENTAT_GATE_MAXK 8
typedef struct mentat_gate_params {
    double temperature;     /* entropy temperature (generator.py:342) */
    double penalty;         /* repetition penalty (generator.py:363-366) */
    double alpha;           /* entropy EMA alpha (generator.py:349) */
    double mult;            /* relative_entropy_multiplier (generator.py:352) */
    double initial;         /* soft_explore_initial (generator.py:331) */
    int32_t K;              /* branching factor, <= MENTAT_GATE_MAXK */
    int32_t M;              /* max_active_branches */
    int32_t num_active;     /* active leaves at the start of the step */
    int32_t step;           /* decode step */
    int32_t window;         /* soft_explore_window */
    int32_t flags;          /* MENTAT_GATE_* bits, 0 by default */
} mentat_gate_params;
/* flags: leave pen_entropy out (0 in the record).  The reference computes it only
 * for its branch-point diagnostics (generator.py:291-293), not for a decision. */
#define MENTAT_GATE_SKIP_PEN_ENTROPY 1
/* flags: log-softmax as (x - max) - log(S) with log(S) in float and one rounding,
 * which is how torch's CUDA kernels compute it; the default rounds log(S) to the
 * logits dtype first, as torch's CPU kernels do (the rounding chain the golden
 * fixtures pin).  Both are the reference's own arithmetic on its two devices. */
#define MENTAT_GATE_FLOAT_LOGSUM 2

typedef struct mentat_gate_out {
    double entropy;         /* compute_entropy(logits, T), reduced-precision rounding chain */
    double entropy_acc;     /* float-accurate entropy of softmax(logits / T) */
    double pen_entropy;     /* compute_entropy(penalised) at T = 1 (generator.py:293) */
    double ema;             /* updated entropy EMA */
    double tau;             /* branch threshold */
    int32_t branch;         /* 1 = branch (top-K), 0 = extend (argmax) */
    int32_t argmax;
    float argmax_lp;
    int32_t topk_ids[MENTAT_GATE_MAXK];
    float topk_lps[MENTAT_GATE_MAXK];
    int32_t pad[3];
} mentat_gate_out;

/* logits: [n][vocab] (row stride in elements), dtype of the model.
 * hist_ptr/hist_ids: CSR of each leaf's generated token ids (duplicates allowed).
 * ema_old: device double[n]; NaN means "no EMA yet" (TreeNode.entropy_ema None).
 * out: device mentat_gate_out[n]. */
int mentat_gate_step(const void* logits, int32_t dtype, int32_t n, int32_t vocab,
                     int64_t row_stride, const int32_t* hist_ptr, const int32_t* hist_ids,
                     const double* ema_old, const mentat_gate_params* params,
                     mentat_gate_out* out, cudaStream_t s);

/*
 * Semantic diversity pruning, pair resolution.  Replaces the masking, the
 * nonzero().tolist() and the host loop of MentatGenerator._prune_similar
 * (generator.py:446-484); the similarity matrix itself is the caller's
 * F.normalize + torch.mm (:441-444).  The leaves of ngroups trees are laid out
 * tree after tree: tree g owns rows/columns group_off[g] .. group_off[g+1]-1 of
 * sim ([m][m] of dtype, row stride sim_stride elements; entries between trees
 * are not read), each tree at most max_group <= 4096 leaves.  parent_key: equal
 * for siblings (the same parent), distinct otherwise; logp: each leaf's
 * cumulative log-prob (double); threshold: the similarity threshold rounded to
 * dtype (torch compares the product in the matrix's dtype).  prune_out: one byte
 * per leaf, 1 for the leaves the reference's loop prunes.
 */
int mentat_prune_similar(const void* sim, int32_t dtype, int64_t sim_stride, const int32_t* group_off,
                         int32_t ngroups, int32_t max_group, const int64_t* parent_key, const double* logp,
                         float threshold, uint8_t* prune_out, cudaStream_t s);

#ifdef __cplusplus
}
#endif
#endif /* MENTAT_B200_H */

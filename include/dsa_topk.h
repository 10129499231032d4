/*
 * dsa_topk.h — C ABI of the B200 (sm_100a) DSA top-k page-table transform
 * (libdsa_topk.so).
 *
 * The library replaces the device work behind the reference operator
 *   dsa_topk_page_table_transform(scores, page_table, q_pos, kv_lens,
 *                                 out_blocks, out_pages, block_size, top_k)
 * in src/task02_dsa_topk_page_table_transform.py:1666-1726 of
 * sinpeyw/flagos-kernelgen-72h-shanghai-2026, i.e. the Triton kernels its
 * NVIDIA routing picks (:1685-1712, :771-817, :955-1216). All of them compute
 * the same per-row selection; one kernel here covers every shape.
 *
 * Per row r = (b, h, q) of scores [B, H, Q, NB] (row-major, r = (b*H+h)*Q+q):
 *   pos  = int32(q_pos[b*Q + q]),  kv = int32(kv_lens[b])
 *   last = min(pos / block_size, min(ceil(kv / block_size), NB) - 1)
 *   block i is a candidate iff pos >= 0 and i <= last, and selectable iff
 *   also its score (as fp32) is not -inf
 *   order: the score's order-preserving key (-0.0 == +0.0) descending, then
 *          the block id ascending (exact, whatever the ties)
 *   out_blocks[r, k] = id of the k-th selectable block in that order, or -1
 *   out_pages[r, k]  = page_table[b*NB + that id], or -1
 *
 * Memory contract: destination passing; every pointer is a device pointer the
 * caller owns, all tensors contiguous. Nothing is allocated and no scratch
 * memory is used. The launch is asynchronous on the given stream.
 */
#ifndef DSA_TOPK_H
#define DSA_TOPK_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DSA_TOPK_ABI_VERSION 1

enum dsa_topk_dtype {
    DSA_DTYPE_FP32 = 0,
    DSA_DTYPE_BF16 = 1,
    DSA_DTYPE_FP16 = 2,
    DSA_DTYPE_INT32 = 3,
    DSA_DTYPE_INT64 = 4
};

enum dsa_topk_status {
    DSA_OK = 0,
    DSA_ERR_NULL_POINTER = 1,   /* a required pointer is NULL                   */
    DSA_ERR_BAD_SHAPE = 2,      /* B, H, Q < 0, NB < 1, NB % 4, block_size < 1   */
    DSA_ERR_BAD_TOPK = 3,       /* top_k < 1 or > 2048                           */
    DSA_ERR_BAD_DTYPE = 4,      /* unsupported dtype                             */
    DSA_ERR_ALIGNMENT = 5,      /* scores not 16-byte aligned, or an index tensor
                                   not aligned to its element size               */
    DSA_ERR_UNSUPPORTED = 6,    /* NB > 16384, or B*H*Q >= 2^31                  */
    DSA_ERR_CUDA = 7,           /* a CUDA runtime call failed                    */
    DSA_ERR_BAD_ARGS_SIZE = 8   /* struct_size mismatch or reserved field not 0  */
};

/*
 * Arguments of one call; replaces the positional arguments of the reference
 * operator (task02…py:1666). Extensions: dtypes of the index tensors are
 * explicit (the reference loads whatever the tensors hold and casts q_pos and
 * kv_lens to int32, :161-162).
 */
typedef struct dsa_topk_args {
    uint32_t struct_size;        /* = sizeof(dsa_topk_args_t)                     */
    int32_t  scores_dtype;       /* FP32 | BF16 | FP16                            */
    int32_t  index_dtype;        /* INT32 | INT64: q_pos and kv_lens              */
    int32_t  page_dtype;         /* INT32 | INT64: page_table and out_pages       */
    int32_t  blocks_dtype;       /* INT32 | INT64: out_blocks                     */
    int32_t  block_size;         /* tokens per KV block, >= 1                     */
    int32_t  top_k;              /* K, 1..2048                                    */
    int32_t  reserved0;          /* must be 0                                     */
    int64_t  B, H, Q, NB;        /* scores [B, H, Q, NB]; NB % 4 == 0, <= 16384   */
    const void* scores;          /* [B, H, Q, NB]                                 */
    const void* page_table;      /* [B, NB]                                       */
    const void* q_pos;           /* [B, Q]                                        */
    const void* kv_lens;         /* [B]                                           */
    void*    out_blocks;         /* [B, H, Q, K]                                  */
    void*    out_pages;          /* [B, H, Q, K]                                  */
} dsa_topk_args_t;

/*
 * Launch the transform on `stream` (a cudaStream_t; NULL = legacy default
 * stream) of the current device. Validates every argument first and returns
 * a dsa_topk_status; on DSA_OK the work is queued, not finished.
 * Replaces: dsa_topk_page_table_transform, task02…py:1666-1726.
 */
int dsa_topk_launch(const dsa_topk_args_t* args, void* stream);

/* Static string for a dsa_topk_status (never NULL). No reference
 * counterpart: the reference raises whatever Triton raises. */
const char* dsa_topk_strerror(int status);

/* DSA_TOPK_ABI_VERSION of the loaded library. No reference counterpart. */
int dsa_topk_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* DSA_TOPK_H */

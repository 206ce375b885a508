/*
 * moe_b200.h -- C ABI of the B200 fused-MoE expert engine.
 *
 * Plain pointers and sizes only: device pointers are CUDA device addresses,
 * `stream` is a cudaStream_t passed as void*.  Every entry point returns
 * MOE_OK (0) or a negative status; moe_last_error() gives the message of the
 * last failure on the calling thread.  Nothing throws across this boundary.
 *
 * Each declaration names the reference interface it replaces
 * (Qeeweew/MoE-Ascend-Opt, paths relative to that project).
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_OK 0
#define MOE_ERR_INVALID (-1)   /* bad argument: shape, dtype, pointer, size */
#define MOE_ERR_CUDA (-2)      /* a CUDA runtime call failed */
#define MOE_ERR_STATE (-3)     /* call not valid in the engine's state (e.g. no weights) */
#define MOE_ERR_DEVICE (-4)    /* a kernel reported an error (bounded wait expired) */

/* quant formats: Int8-gemm/quant_traits.h:7-10 (Q8_0 = 0, Q4_0 = 1); AWQ W4A16 is new. */
#define MOE_Q8_0 0
#define MOE_Q4_0 1
#define MOE_AWQ 2

/* element types of activations, scales and weight inputs */
#define MOE_F16 0
#define MOE_BF16 1
#define MOE_F32 2

typedef struct moe_engine moe_engine;

typedef struct moe_config {
    int64_t num_experts;       /* experts held by this engine (E, or E/ep_size under EP) */
    int64_t hidden_size;       /* H, multiple of 32 (of the AWQ group for AWQ) */
    int64_t intermediate_size; /* I, multiple of 32 (of the AWQ group for AWQ) */
    int32_t quant_type;        /* MOE_Q8_0 / MOE_Q4_0 / MOE_AWQ */
    int32_t group_size;        /* AWQ group along K (128); ignored otherwise */
    int32_t device;            /* CUDA device ordinal */
    int32_t expert_offset;     /* global id of this engine's first expert (EP); 0 otherwise */
} moe_config;

/* Replaces MoEInfer::MoEInfer (Int8-gemm/moe_infer.cpp:18-75) and the
 * MoEInfer torch class constructor (Int8-gemm/nanovllm_ops.cpp:23-31).
 * Checks H % 32 == 0 and I % 32 == 0 as the reference does (moe_infer.cpp:27-31). */
int moe_engine_create(const moe_config* cfg, moe_engine** out);
/* Replaces MoEInfer::~MoEInfer (Int8-gemm/moe_infer.cpp:77-84). */
int moe_engine_destroy(moe_engine* eng);

/* Replaces MoEInfer::store_quantized_weights_repack (Int8-gemm/moe_infer.cpp:96-282).
 * Row-major input contract (host or device memory, src_on_device says which):
 *   Q8_0: gate_up_qs int8 [E,2I,H], down_qs int8 [E,H,I]
 *   Q4_0: gate_up_qs uint32 [E,2I,H/8], down_qs uint32 [E,H,I/8], element k of a row
 *         at word k/8, bits 4*(k%8), value nibble-8
 *   scales gate_up_d [E,2I,H/32], down_d [E,H,I/32], both MOE_F16 or both MOE_BF16.
 * Rows [0,I) of gate_up are gate_proj, rows [I,2I) up_proj. */
int moe_engine_load_quantized(moe_engine* eng, const void* gate_up_qs, const void* gate_up_d,
                              const void* down_qs, const void* down_d, int32_t scale_dtype,
                              int32_t src_on_device, void* stream);

/* Replaces MoEInfer::quantize_and_store_expert (Int8-gemm/moe_infer.cpp:284-360) with
 * quantize_weight_only (Int8-gemm/q8_gemm.cpp:219-260): Q8_0 only, fp16 scales.
 * proj: 0 = gate_proj [I,H], 1 = up_proj [I,H], 2 = down_proj [H,I];
 * w_dtype MOE_F32 / MOE_F16 / MOE_BF16. */
int moe_engine_quantize_store_expert(moe_engine* eng, int64_t expert, int32_t proj, const void* w,
                                     int32_t w_dtype, int32_t src_on_device, void* stream);

/* AWQ W4A16 weights (no reference counterpart in this checkout: the Ascend
 * grouped_gemv kernel of sgl-kernel-npu is absent).  AutoAWQ GEMM packing:
 *   w13_qweight int32 [E, H, 2I/8], w13_scales bf16 [E, H/G, 2I], w13_qzeros int32 [E, H/G, 2I/8]
 *   w2_qweight  int32 [E, I, H/8],  w2_scales  bf16 [E, I/G, H],  w2_qzeros  int32 [E, I/G, H/8]
 * 8 values per int32 in the AWQ order {0,2,4,6,1,3,5,7}; W = (q - z) * s. */
int moe_engine_load_awq(moe_engine* eng, const void* w13_qweight, const void* w13_scales,
                        const void* w13_qzeros, const void* w2_qweight, const void* w2_scales,
                        const void* w2_qzeros, int32_t src_on_device, void* stream);

/* Replaces MoEInfer::execute_on_cpu_routed_from_pointers (Int8-gemm/moe_infer.cpp:430-456)
 * -> moe_forward_ptr_impl (Int8-gemm/q8_gemm.cpp:276-646).  All pointers on the engine's
 * device: x [T,H] (act_dtype), y [T,H] (out_dtype: act_dtype, or MOE_F32 for a partial
 * sum under expert parallelism), topk_ids int32 [T,K], topk_w fp32 [T,K].  Ids outside
 * this engine's experts are skipped (moe_common.cpp:158,175-181).  Stream ordered. */
int moe_engine_forward(moe_engine* eng, const void* x, void* y, const int32_t* topk_ids,
                       const float* topk_w, int64_t num_tokens, int64_t top_k, int32_t act_dtype,
                       int32_t out_dtype, void* stream);

/* Dense MLP (a shared expert, or a dense FFN layer) through the same fused kernels:
 * y = down(SiLU(gate x) * up x) of local expert `expert` for every token, i.e.
 * moe_engine_forward with top_k = 1, that expert and weight 1 (the routing is kept in an
 * engine buffer, allocated on the first call with more tokens than before).  A shared expert
 * fuses into the routed layer without this call: load it as one more expert and pass its id
 * as an extra top-k column with its gate weight (1, or the model's shared-expert gate).
 * No counterpart in the reference, whose engine only serves routed experts. */
int moe_engine_forward_dense(moe_engine* eng, int64_t expert, const void* x, void* y, int64_t num_tokens,
                             int32_t act_dtype, int32_t out_dtype, void* stream);

/* Reserve the forward's device workspace for up to max_tokens x top_k so that
 * later forwards allocate nothing (needed before CUDA graph capture).
 * Replaces the role of NumaBufferPool::ensure_capacity (Int8-gemm/moe_common.cpp:57-111). */
int moe_engine_reserve(moe_engine* eng, int64_t max_tokens, int64_t top_k);

/* Device time of the last forward in ms (CUDA events on the forward's stream; waits for
 * it).  Replaces MoEInfer::get_last_run_time_ms (Int8-gemm/moe_infer.h:24). */
int moe_engine_last_time_ms(moe_engine* eng, double* ms);

/* Reads and clears the device error word of the engine's workspace (waits for the device).
 * *code = 0 when every kernel completed; non-zero when a bounded wait expired. */
int moe_engine_device_error(moe_engine* eng, int32_t* code);

/* Decode the engine's device-resident weights of one expert back into row-major form
 * (bit-exact check of the load-time packing).  which: 0 gate_up (2I rows of H), 1 down
 * (H rows of I).  Q8_0/Q4_0: qs_out / d_out receive the input-contract rows.  AWQ: qs_out
 * receives per row the K/2 bytes of sequential nibbles (element k at byte k/2, low nibble
 * for even k), d_out per row the K/G bf16 scales followed by the K/G zero points (u8). */
int moe_engine_export_expert(moe_engine* eng, int64_t expert, int32_t which, void* qs_out,
                             void* d_out);

/* Router (Int8-gemm/test/fused_moe_cpu.py:20-37): top-K of fp32 logits [T,E] in
 * descending order (ties: lower expert id first), weights = softmax over the K selected
 * logits (renormalize != 0) or softmax over all E gathered at the selection. */
int moe_route_topk(const float* logits, int64_t num_tokens, int64_t num_experts, int64_t top_k,
                   int32_t renormalize, int32_t* topk_ids, float* topk_w, void* stream);

/* Router GEMM fused with the top-k of moe_route_topk: logits[t][e] = sum_h hidden[t][h] *
 * router_w[e][h] (fp32 accumulate), then the selection and weights of moe_route_topk.  The
 * reference computes the router logits outside its op and routes with
 * Int8-gemm/test/fused_moe_cpu.py:20-37; this entry point is the attention-side pre-step
 * that feeds moe_engine_forward directly.  hidden [T,H] (act_dtype MOE_F16 / MOE_BF16),
 * router_w [E,H] (MOE_F16 / MOE_BF16 / MOE_F32), H a multiple of 8; logits [T,E] fp32 is
 * written when non-null.  Device pointers, stream ordered. */
int moe_route_gemm_topk(const void* hidden, int32_t act_dtype, const void* router_w, int32_t w_dtype,
                        int64_t num_tokens, int64_t hidden_size, int64_t num_experts, int64_t top_k,
                        int32_t renormalize, int32_t* topk_ids, float* topk_w, float* logits, void* stream);

/* Stable counting sort of routed pairs by expert (Int8-gemm/moe_common.cpp:146-216):
 * counts [E], starts [E+1], token_map [T*K][2] = (t,k) per position, scatter_map [T*K]
 * (-1 for ids outside [0,E)).  Device pointers. */
int moe_route_permute(const int32_t* topk_ids, int64_t num_tokens, int64_t top_k,
                      int64_t num_experts, int32_t* counts, int32_t* starts, int32_t* token_map,
                      int32_t* scatter_map, void* stream);

/* Q8_0 activation quantisation of rows (Int8-gemm/gemm_kernels.cpp:25-58, stage A of
 * Int8-gemm/q8_gemm.cpp:360-377): x [rows, cols] (dtype) -> qs int8 [rows, cols],
 * d fp32 [rows, cols/32].  Device pointers. */
int moe_quantize_rows_q8_0(const void* x, int32_t dtype, int64_t rows, int64_t cols, int8_t* qs,
                           float* d, void* stream);

/* Diagnostics (no counterpart in the reference): enable != 0 makes every later decode
 * launch record 20 stamps per CTA (globaltimer ns unless noted).  Persistent decode kernels
 * (one row per SM): phase boundaries of the fused kernel: start, routing, activation
 * quantisation, first/last gate_up data, gate_up done, grid barrier entered/passed, h
 * requantised, first down data, down done, combine done, SM clock at start/end, first down
 * issue (split-K kernel: its chunk count and h slots), barrier arrival fenced/observed, warp 0
 * down loop done / first down wait.  Two-pass kernels (one row per CTA of the grid, row =
 * slot x tiles + tile; pass 1 in entries 0-9: start, dependency wait passed, routed and
 * tokens staged, weight copies issued, [AWQ: weight data], end; pass 2 in entries 10-19: start,
 * routed, copies issued, dependency wait passed, h staged, weight data, dots done, arrival,
 * combine done).  Rows beyond the buffer's (at least 1024) are not recorded.
 * enable == 0 turns it off.  When `out` is non-null, copies up to max_entries stamps of
 * the last launch (waits for the device).  *n_entries = rows x 20 while enabled. */
int moe_engine_debug_timeline(moe_engine* eng, int32_t enable, uint64_t* out, int32_t max_entries,
                              int32_t* n_entries);

/* Forward that allocates nothing (no counterpart in the reference).  For callers that may
 * not call cudaMalloc when they run the layer -- serving runtimes that reserve the whole
 * device memory at start-up and forbid later allocations, or latency-critical paths that
 * cannot afford an allocation's implicit device synchronisation.  Same arguments and result
 * as moe_engine_forward, on an engine whose weights are loaded; its scratch comes from a
 * fixed 512 KiB array in device memory that every GPU loading this library holds until the
 * process exits.  Limit: 256 + 4*T*K*I bytes must fit in 512 KiB (e.g. T*K <=
 * 170 at I = 768) and T must fit one decode launch; larger calls fail with MOE_ERR_INVALID.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture.  All calls share the one array: calls
 * that overlap on the GPU (other streams, other threads) race and must be serialised. */
int moe_engine_forward_noalloc(moe_engine* eng, const void* x, void* y, const int32_t* topk_ids,
                               const float* topk_w, int64_t num_tokens, int64_t top_k,
                               int32_t act_dtype, int32_t out_dtype, void* stream);

/* Packed-layout files (no counterpart in the reference, whose engine repacks every load:
 * MoEInfer::store_quantized_weights_repack, Int8-gemm/moe_infer.cpp:96-282).
 * moe_engine_save writes the engine's device-resident weight layouts (all formats, after any
 * load call) with a header of the shape, format and record sizes and a checksum per section;
 * moe_engine_load_file fills an engine created with the same moe_config from such a file by
 * plain copies (no repacking) and fails with MOE_ERR_INVALID on a different shape or format,
 * a truncated file or a checksum mismatch.  Both synchronise the device. */
int moe_engine_save(moe_engine* eng, const char* path);
int moe_engine_load_file(moe_engine* eng, const char* path);

/* Message of the last failed call on this thread ("" if none). */
const char* moe_last_error(void);

/* Expert-parallel combine over peer memory (no counterpart in the reference, whose NUMA
 * "TP" nodes reduce into node 0, q8_gemm.cpp:621-641).  One process per GPU; rank r's
 * engine holds experts [r*E/W, (r+1)*E/W) (moe_config.expert_offset).  Each rank creates a
 * mailbox for `world` ranks and up to min(max_tokens, 64) tokens per decode launch and gets
 * its CUDA IPC handle (64 bytes) back; the caller exchanges the handles (e.g. an all-gather)
 * and passes all of them, in rank order, to moe_engine_p2p_connect.  From then on,
 * moe_engine_forward calls that take the fused decode kernels sum the ranks' partials
 * inside the kernel (NVLink stores into every rank's mailbox, per-CTA flags, bounded
 * waits) and write the full output on every rank; all ranks must make the same sequence
 * of such calls.  While connected, calls that moe_engine_p2p_covers() rejects (the
 * grouped-GEMM sizes) fail with MOE_ERR_STATE: disable the combine with
 * moe_engine_p2p_enable(eng, 0), run the layer with MOE_F32 output (this rank's partial) and
 * all-reduce it, then enable it again.  A peer that does not arrive within about a second
 * sets device error 4 (moe_engine_device_error). */
int moe_engine_p2p_mailbox(moe_engine* eng, int32_t world, int64_t max_tokens, void* ipc_handle_out);
int moe_engine_p2p_connect(moe_engine* eng, int32_t rank, int32_t world, const void* ipc_handles);
int moe_engine_p2p_enable(moe_engine* eng, int32_t on);
int moe_engine_p2p_covers(moe_engine* eng, int64_t num_tokens);

/* Expert placement for load balance under skewed routing (the reference places experts
 * on NUMA nodes in contiguous blocks, moe_infer.cpp:143-205).  Replaces the contiguous block
 * [expert_offset, expert_offset + num_experts) by an explicit map: local_of_global[g] is
 * the local index (0 .. num_experts-1) of global expert g on this engine, or -1 when another
 * engine holds it; every local index appears once.  The weights loaded into local slot l
 * must be those of the global expert mapped to l.  An entry `l | MOE_REPLICATED` marks a hot
 * expert that every rank holds (replication of hot experts): this engine then computes its
 * routed pairs only for tokens t with (t + g) % world == rank, from moe_engine_set_replica_split,
 * so that each pair is computed once across the ranks.  Copied to the device (synchronises). */
#define MOE_REPLICATED (1 << 30)
int moe_engine_set_expert_map(moe_engine* eng, const int32_t* local_of_global, int64_t num_global);
/* This engine's rank and the world size for the replicated experts of its map (default 0 of 1). */
int moe_engine_set_replica_split(moe_engine* eng, int32_t rank, int32_t world);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */

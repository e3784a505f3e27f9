/*
 * engram_b200.h -- C ABI of the B200 (sm_100a) Engram/PLE table path.
 *
 * The reference (fulvian/engraft-ngram) is Python; the FFI it would bind for
 * this path is ctypes (engraft_ngram_b200/_lib.py is that binding).  Every
 * entry point:
 *   - takes plain pointers and sizes (device pointers unless noted "host");
 *   - is enqueued on the caller's CUDA stream (`stream`, a cudaStream_t; NULL =
 *     the legacy default stream), makes no host synchronisation and allocates
 *     no memory (scratch space is passed in);
 *   - returns 0 on success or a negative ENGRAM_ERR_* code; nothing is launched
 *     when an argument check fails.
 *
 * Reference interfaces replaced (paths inside the reference project):
 *   engram_table_init / engram_table_pack  <- PleTable.__init__ + read_rows_raw
 *       (engraft/table.py:48-104): the table's addressing constants, and the
 *       per-head IQ4_NL rows made resident in HBM instead of read per row.
 *   engram_hash            <- PleTable.ngram_addresses (engraft/table.py:111-144),
 *       damage.ngram_rows (engraft/damage.py:68-104), lens.local_to_global
 *       (engraft/lens.py:108-110).
 *   engram_overlay_map_build <- the row_map dict membership test
 *       (engraft/replica/seq.py:401-417, engraft/replica/distill.py:401-457).
 *   engram_forward         <- OverlayEmb.build (engraft/replica/seq.py:372-444) with
 *       RowSet.from_position + dequant_iq4nl (engraft/lens.py:127-136,
 *       engraft/table.py:147-169) and dequant_iq4_xs (engraft/replica/dequant.py:150-189).
 *   engram_backward        <- autograd of rows_var[idx_r] / index_put
 *       (engraft/replica/seq.py:433-441): row gradients, duplicates summed.
 *   engram_adam_step       <- reg.backward() + torch.optim.Adam.step()
 *       (engraft/descend_corpus.py:921-947).
 */
#ifndef ENGRAM_B200_H
#define ENGRAM_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define ENGRAM_API __attribute__((visibility("default")))
#else
#define ENGRAM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
#define ENGRAM_OK 0
#define ENGRAM_ERR_ARG (-1)       /* null pointer, negative size, bad enum      */
#define ENGRAM_ERR_FORMAT (-2)    /* unsupported fmt / dim / mode combination   */
#define ENGRAM_ERR_RANGE (-3)     /* table geometry or a size out of range      */
#define ENGRAM_ERR_WORKSPACE (-4) /* scratch buffer too small                   */
#define ENGRAM_ERR_CUDA (-5)      /* a launch failed (cudaGetLastError)         */

/* ---- row formats of the resident table ---------------------------------- */
#define ENGRAM_FMT_F32 0    /* dim floats per row                              */
#define ENGRAM_FMT_IQ4_NL 1 /* ggml IQ4_NL, dim/32 blocks (the reference table) */
#define ENGRAM_FMT_IQ4_XS 2 /* ggml IQ4_XS, dim/256 superblocks                 */

/* ---- output modes of engram_forward ------------------------------------- */
/* out float [n, n_heads, dim]: the reference's emb (row h of position t at
 * out[t, h, :], engraft/replica/seq.py:444 reshapes it to [n, n_heads*dim]).  */
#define ENGRAM_MODE_CONCAT_F32 0
/* out bf16 [n, heads_per_ngram*dim], updated in place:
 *   out[t, g*dim+c] = bf16_rn(float(out[t, g*dim+c]) + (row[g][c] + row[hpn+g][c]))
 * i.e. the bigram and trigram rows of group g summed into the residual stream.
 * Builder-defined; requires ngram_size == 3.                                  */
#define ENGRAM_MODE_PAIRSUM_ADD_BF16 1

#define ENGRAM_MAX_HEADS 32
#define ENGRAM_MAX_CTX 4

/*
 * Table descriptor, filled by engram_table_init.  Plain data in host memory,
 * owned by the caller; passed by pointer and copied by value into launches.
 */
typedef struct engram_table {
    const void* rows;      /* device, resident rows (layout: engram_table_pack) */
    int64_t n_rows;
    int64_t row_stride;    /* bytes between rows                               */
    int32_t fmt;
    int32_t dim;
    int32_t ngram_size;    /* context length N (2..ENGRAM_MAX_CTX)             */
    int32_t heads_per_ngram;
    int32_t n_heads;       /* (N-1) * heads_per_ngram                          */
    int32_t reserved;
    int64_t eos_token_id;
    uint64_t mult[ENGRAM_MAX_CTX];              /* layer_multipliers[0..N-1]  */
    uint64_t head_magic[ENGRAM_MAX_HEADS];      /* x % p_h by multiplication   */
    uint32_t head_size[ENGRAM_MAX_HEADS];       /* p_h                        */
    uint32_t head_shift[ENGRAM_MAX_HEADS];
    int64_t head_offset[ENGRAM_MAX_HEADS];      /* head_offsets[h]            */
} engram_table;

/*
 * Overlay descriptor: the trainable rows and the device map global id -> slot
 * built by engram_overlay_map_build.  R == 0 means "no overlay".
 */
typedef struct engram_overlay {
    const float* rows;      /* device [R, dim] fp32 (rows_var)                 */
    int64_t n_rows;         /* R                                               */
    const int32_t* map_keys;  /* device [capacity]; -1 = empty                 */
    const int32_t* map_slots; /* device [capacity]                             */
    int64_t capacity;       /* power of two >= 2R (0 when R == 0)              */
} engram_overlay;

/* dim: 1..1024; F32 needs dim % 4 == 0 (dim % 8 == 0 for PAIRSUM_ADD_BF16),
 * IQ4_NL dim % 32 == 0, IQ4_XS dim % 256 == 0. */

/* Bytes per resident row: F32 dim*4; IQ4_NL round_up(dim/32*18, 16);
 * IQ4_XS dim/256*144.  Negative on an unsupported fmt/dim.                    */
ENGRAM_API int64_t engram_row_stride(int32_t fmt, int32_t dim);

/* Bytes per row of the reference's own (GGUF) layout: F32 dim*4; IQ4_NL
 * dim/32*18; IQ4_XS dim/256*136.                                              */
ENGRAM_API int64_t engram_raw_row_bytes(int32_t fmt, int32_t dim);

/*
 * Fills *t (host memory).  head_sizes/head_offsets/mult are HOST arrays of
 * n_heads = (ngram_size-1)*heads_per_ngram, n_heads and ngram_size entries
 * (mult may hold more; the first ngram_size are used).  Checks 1 <= p_h,
 * head_offsets[h] + p_h <= n_rows <= 2^31-1, and computes the per-head
 * division magic (Granlund & Montgomery, PLDI 1994, unsigned case).
 * Replaces PleTable.__init__ (engraft/table.py:48-88).
 */
ENGRAM_API int engram_table_init(engram_table* t, const void* rows, int64_t n_rows, int32_t fmt, int32_t dim,
                      int32_t ngram_size, int32_t heads_per_ngram, const int64_t* head_sizes,
                      const int64_t* head_offsets, const uint64_t* mult, int32_t n_mult,
                      int64_t eos_token_id);

/*
 * Repacks rows from the reference's layout (src: device, n_rows *
 * engram_raw_row_bytes) into the resident layout (dst: device, n_rows *
 * engram_row_stride).  Resident layouts (16-byte aligned rows):
 *   F32:    unchanged.
 *   IQ4_NL: [qs of the dim/32 blocks, 16 B each][fp16 d of each block][zero pad].
 *   IQ4_XS: per superblock 144 B = [qs 128 B][d 2 B][scales_h 2 B][scales_l 4 B][8 zero B].
 * Replaces PleTable.read_rows_raw (engraft/table.py:90-104) as the row source.
 */
ENGRAM_API int engram_table_pack(int32_t fmt, int32_t dim, const uint8_t* src, int64_t n_rows, void* dst, void* stream);

/*
 * Builds the open-addressing map global id -> slot for the overlay rows:
 * map[ids[k]] = k.  keys/slots: device [capacity], capacity a power of two
 * >= 2R; the kernel clears them first.  ids must be distinct and >= 0 (the
 * keys of the reference's row_map, engraft/replica/distill.py:452-453).
 */
ENGRAM_API int engram_overlay_map_build(const int32_t* ids, int64_t R, int32_t* keys, int32_t* slots,
                             int64_t capacity, void* stream);

/*
 * Overlay membership of a batch of global ids: slots_out[k] = row_map[ids[k]]
 * or -1 (the reference's `g in row_map`, engraft/replica/seq.py:411-417).
 */
ENGRAM_API int engram_overlay_lookup(const engram_overlay* ov, const int32_t* ids, int64_t n, int32_t* slots_out,
                                     void* stream);

/*
 * K1 alone: global row ids [n, n_heads] (int32) of positions t0..t0+n-1 of
 * `tokens` (device int32; tokens before t0 are read as context).  seg_start
 * (device int32 [t0+n] or NULL): seg_start[t] = first index of t's segment;
 * a predecessor before it counts as missing (engraft/replica/seq.py:393-399).
 * Bit-identical to PleTable.ngram_addresses + local_to_global.
 */
ENGRAM_API int engram_hash(const engram_table* t, const int32_t* tokens, const int32_t* seg_start, int64_t t0,
                int64_t n, int32_t* ids_out, void* stream);

/*
 * Fused hash -> overlay lookup -> gather/dequant -> emit, one launch.
 * out: see ENGRAM_MODE_*.  ids_out (nullable) int32 [n, n_heads] global ids;
 * slots_out (nullable) int32 [n, n_heads] overlay slot or -1 (the input of
 * engram_backward); hit_count (nullable) device int64[1] += number of
 * (position, head) pairs served by the overlay (OverlayEmb.n_id_hits).
 */
ENGRAM_API int engram_forward(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                   const int32_t* seg_start, int64_t t0, int64_t n, int32_t mode, void* out,
                   int32_t* ids_out, int32_t* slots_out, int64_t* hit_count, void* stream);

/*
 * engram_forward with the table rows taken from a gathered buffer: t->rows
 * points at rows laid out like the resident table (t->row_stride bytes each)
 * and row_index (device int32 [n, n_heads]) gives, for each (output row, head),
 * the row to read; entries for heads the overlay serves are ignored (-1).
 * The hash and the overlay probe still use t's addressing constants, so ids_out,
 * slots_out and hit_count are those of engram_forward.  Used by the row-sharded
 * table after the all-to-all of rows (engram_shard_requests / _gather).
 */
ENGRAM_API int engram_forward_indirect(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                       const int32_t* seg_start, int64_t t0, int64_t n, const int32_t* row_index,
                                       int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                                       int64_t* hit_count, void* stream);

/*
 * engram_forward over a row-sharded table read in place: row g lives at local
 * row g / world of rank (g % world)'s shard, and shard_rows (device array
 * [world] of pointers valid in this process, e.g. each rank's shard in torch
 * symmetric memory, mapped over NVLink) gives each shard's first row.  The
 * kernels copy each row straight from its owner's memory (peer loads), so no
 * exchange step runs before the forward.  t supplies the addressing constants
 * of the whole table (n_rows = all rows); its rows pointer is not read.  No
 * reference counterpart: the reference is single-process.
 */
ENGRAM_API int engram_forward_sharded(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                      const int32_t* seg_start, int64_t t0, int64_t n, const void* shard_rows,
                                      int32_t world, int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                                      int64_t* hit_count, void* stream);

/*
 * The sharded forward in two launches that can run apart: the rows of other
 * ranks are copied ahead into this GPU's memory (the table shards never
 * change, so the copy for the next batch can overlap the current step on a
 * side stream), then the forward reads every row locally.
 *
 * engram_stage_bytes: bytes of `stage` for n output rows (n * n_heads *
 * row_stride).
 * engram_stage_sharded: for output rows [0, n) of positions t0.., head h of
 * row i with owner g % world != rank is copied to stage + (i * n_heads + h) *
 * row_stride (16-byte aligned); this rank's rows are not copied, nor are the
 * heads the overlay ov serves (nullable; only its map is read, and it must be
 * the map the forward uses).  max_blocks caps the grid (0: the whole GPU).
 * world == 1 copies nothing.
 * engram_forward_staged: engram_forward_sharded reading rank's own rows in
 * place and every other row from `stage`, which must hold the copy made for
 * the same tokens, seg_start, t0 and n (ordered before this call).  Outputs
 * are bit-identical to engram_forward_sharded.  No reference counterpart.
 */
ENGRAM_API int64_t engram_stage_bytes(const engram_table* t, int64_t n);
ENGRAM_API int engram_stage_sharded(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                    const int32_t* seg_start, int64_t t0, int64_t n, const void* shard_rows,
                                    int32_t world, int32_t rank, void* stage, int32_t max_blocks, void* stream);
/*
 * Push staging, the collective form of the staged sharded read (world <= 16).
 * Each rank's stage holds every row its forward reads, grouped by owner
 * (block o = the rows rank o owns, in output-row-then-head order), so every
 * owner writes each requester's block as contiguous NVLink stores; the forward
 * is engram_forward_indirect with rows = the stage and row_index below.
 *
 * engram_stage_plan_words: int32 entries of a plan, world * (ceil(n/32) + 1).
 * engram_stage_plan (requester, local): plan[o * (tiles + 1) + k] = stage row
 *   of the first row of 32-row tile k served by owner o (entry `tiles` = end
 *   of block o); row_index[i * n_heads + h] (n * n_heads int32) = stage row of
 *   head h of output row i.  Every rank's stage then holds n * n_heads rows.
 * engram_stage_push (owner, t->rows = its shard): for every rank r (itself
 *   included) and every tile of r's batch (token_ptrs[r], seg_ptrs[r] or
 *   none, plan_ptrs[r]: device arrays [world] of pointers valid here, e.g.
 *   symmetric memory), the rows this rank owns go to stage_ptrs[r] from row
 *   plan_r[rank][k] on.  The caller orders the ranks around it: every rank's
 *   tokens and plan written and its previous forward over the stage done
 *   before it, a barrier after it before any forward reads its stage.
 * n * n_heads < 2^31.  No reference counterpart.
 */
ENGRAM_API int64_t engram_stage_plan_words(int64_t n, int32_t world);
ENGRAM_API int engram_stage_plan(const engram_table* t, const int32_t* tokens, const int32_t* seg_start, int64_t t0,
                                 int64_t n, int32_t world, int32_t* plan, int32_t* row_index, void* stream);
ENGRAM_API int engram_stage_push(const engram_table* t, const void* token_ptrs, const void* seg_ptrs,
                                 const void* plan_ptrs, int64_t t0, int64_t n, const void* stage_ptrs, int32_t world,
                                 int32_t rank, int32_t max_blocks, void* stream);
ENGRAM_API int engram_forward_staged(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                     const int32_t* seg_start, int64_t t0, int64_t n, const void* shard_rows,
                                     int32_t world, int32_t rank, const void* stage, int32_t mode, void* out,
                                     int32_t* ids_out, int32_t* slots_out, int64_t* hit_count, void* stream);

/*
 * Row-sharded table (owner(g) = g mod world, local index g / world), step 1 of
 * the exchange: from the global ids [n] (n = positions * heads) and the overlay
 * slots (nullable; entries with slot >= 0 need no table row), builds
 *   send_ids  (device int32 [<= n]): the distinct ids, grouped by owner rank;
 *   counts    (device int64 [2*world]): counts[o] = ids for owner o (the rest
 *             is scratch);
 *   row_index (device int32 [n]): position of each entry's id in send_ids
 *             (= its row in the reply), -1 for overlay entries.
 * set_keys/set_vals: device int32 [capacity] scratch, capacity a power of two
 * >= 2n.  The order inside an owner's group is unspecified; results do not
 * depend on it.  No reference counterpart: the reference is single-process.
 */
ENGRAM_API int engram_shard_requests(const int32_t* ids, const int32_t* slots, int64_t n, int32_t world,
                                     int32_t* set_keys, int32_t* set_vals, int64_t capacity, int32_t* send_ids,
                                     int64_t* counts, int32_t* row_index, void* stream);

/*
 * Row-sharded table, the deduplicated exchange plan of one batch: for the
 * (position, head) pairs of positions t0..t0+n-1 of `tokens` (hashed with t's
 * addressing constants, as engram_hash) whose row another rank owns and the
 * overlay ov (nullable; only its map is read) does not serve, builds
 *   send_ids  (device int32 [<= n * n_heads]): the distinct such ids, grouped by
 *             owner (no entry for `rank` itself);
 *   counts    (device int64 [2*world]): counts[o] = ids for owner o; the rest is
 *             scratch;
 *   row_index (device int32 [n * n_heads]): the position of the pair's id in
 *             send_ids (= its row in the reply), -1 for pairs served locally or
 *             by the overlay.
 * set_keys/set_vals: device int32 [capacity] scratch, capacity a power of two
 * >= 2 * n * n_heads.  A Zipf-hot remote row is requested once per batch, not
 * once per occurrence.  No reference counterpart: the reference is
 * single-process.
 */
ENGRAM_API int engram_shard_plan(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                 const int32_t* seg_start, int64_t t0, int64_t n, int32_t world, int32_t rank,
                                 int32_t* set_keys, int32_t* set_vals, int64_t capacity, int32_t* send_ids,
                                 int64_t* counts, int32_t* row_index, void* stream);

/*
 * engram_shard_plan without the deduplication: every (position, head) pair of
 * positions t0..t0+n-1 that another rank owns and the overlay ov (nullable)
 * does not serve requests its row once, grouped by owner in send_ids (the order
 * inside an owner's group is free); counts [2*world] and row_index [n *
 * n_heads] as engram_shard_plan.  Three passes over the pairs and no hash set:
 * cheaper than the plan where few remote rows repeat inside a batch.
 * scratch: device uint32 [engram_shard_route_scratch_words(n, n_heads, world)].
 * No reference counterpart.
 */
ENGRAM_API int64_t engram_shard_route_scratch_words(int64_t n, int32_t n_heads, int32_t world);
ENGRAM_API int engram_shard_route(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                  const int32_t* seg_start, int64_t t0, int64_t n, int32_t world, int32_t rank,
                                  uint32_t* scratch, int64_t scratch_words, int32_t* send_ids, int64_t* counts,
                                  int32_t* row_index, void* stream);

/*
 * engram_forward over a row-sharded table after the exchange of a plan: rows
 * this rank owns are read in place from local_rows (its shard: row g at local
 * row g / world), every other row from recv_rows (the rows of the plan's
 * send_ids, in send order, row_stride bytes each) at the row given by the
 * plan's row_index for the same tokens, seg_start, t0 and n.  t supplies the
 * addressing constants of the whole table; its rows pointer is not read.
 * Outputs are bit-identical to engram_forward on the whole resident table.
 * No reference counterpart.
 */
ENGRAM_API int engram_forward_exchanged(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                        const int32_t* seg_start, int64_t t0, int64_t n, const void* local_rows,
                                        int32_t world, int32_t rank, const void* recv_rows, const int32_t* row_index,
                                        int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out,
                                        int64_t* hit_count, void* stream);

/*
 * The peer-memory exchange with pushed requests (the row-sharded step's
 * default).  Every owner holds, per batch set, a request buffer int32
 * [world][region], a count array int64 [world] and a send buffer of
 * [world][region] rows, all mapped into every rank (e.g. torch symmetric
 * memory); region >= n * n_heads, world * region <= 2^31 - 1.
 *
 * engram_shard_route_push (requester): every (position, head) pair of
 * positions t0..t0+n-1 that another rank owns and the overlay ov (nullable)
 * does not serve sends its id to its owner o: stored in region `rank` of o's
 * request buffer (id_ptrs: device array [world] of pointers valid here, o's
 * request buffer), and the total per owner in entry `rank` of o's count
 * array (count_ptrs, likewise).  counts: device int64 [world], this rank's
 * requests per owner (0 for itself).  row_index [n * n_heads]: the pair's row
 * in the receive buffer, whose blocks follow in ascending owner order (block
 * o = the rows asked of o, counts[o] of them), or -1 for a pair not
 * requested.  The order inside a block is free.  A hashed pair, an owner
 * computation and one store per request: no hash set, no collective.
 *
 * engram_shard_serve_pushed (owner): the rows requester r asked for (ids
 * [0, req_counts[r]) of region r of req_ids, this owner's request buffer) are
 * read from this rank's shard (row g at local row g / world) into region r of
 * send_rows, in the same order, row_stride bytes each; requester r then copies
 * req_counts[r] rows from the start of its region as one transfer.  Ids that
 * are not this rank's give zero rows.  The caller orders every rank's route
 * before any owner's serve, and every owner's serve before any requester's
 * copy (a barrier).  No reference counterpart: the reference is single-process.
 */
ENGRAM_API int engram_shard_route_push(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                       const int32_t* seg_start, int64_t t0, int64_t n, int32_t world, int32_t rank,
                                       const void* id_ptrs, const void* count_ptrs, int64_t region, int64_t* counts,
                                       int32_t* row_index, void* stream);
ENGRAM_API int engram_shard_serve_pushed(const void* shard_rows, int64_t stride, int64_t n_local, int32_t world,
                                         int32_t rank, const int32_t* req_ids, const int64_t* req_counts,
                                         int64_t region, void* send_rows, void* stream);

/*
 * Owner side: out[k] = the resident row of global id ids[k] from this rank's
 * shard (local index ids[k] / world; stride bytes per row, 16-byte multiple).
 * Ids outside the shard give zero rows.
 */
ENGRAM_API int engram_shard_gather(const void* shard_rows, int64_t stride, int64_t n_local, const int32_t* ids,
                                   int64_t n, int32_t world, void* out, void* stream);

/*
 * engram_forward for an explicit list of positions (decode-style lookups: one
 * new token per sequence, each sequence's recent tokens laid out in `tokens`
 * with seg_start marking where each sequence starts).  Output row k is
 * position positions[k] (device int64 [n]; values are clamped into
 * [0, n_tokens)).  Replaces the per-position Replica.ple_true_emb
 * (engraft/replica/model.py:473-495), overlay substituted as there.
 */
ENGRAM_API int engram_forward_at(const engram_table* t, const engram_overlay* ov, const int32_t* tokens,
                                 int64_t n_tokens, const int32_t* seg_start, const int64_t* positions, int64_t n,
                                 int32_t mode, void* out, int32_t* ids_out, int32_t* slots_out, int64_t* hit_count,
                                 void* stream);

/*
 * Dequantised rows by global id: out float [n, dim] = row ids[k] of the table
 * (no overlay).  Replaces distill._read_true_rows (engraft/replica/distill.py:378-396)
 * and PleTable.read_rows (engraft/table.py:106-109) on the resident table.
 * Ids must lie in [0, n_rows); an id outside that range gives a zero row.
 */
ENGRAM_API int engram_gather_rows(const engram_table* t, const int32_t* ids, int64_t n, float* out, void* stream);

/* Scratch bytes engram_backward needs for n positions of n_heads heads and R
 * overlay rows. */
ENGRAM_API int64_t engram_backward_workspace_bytes(int64_t n, int32_t n_heads, int64_t R);

/*
 * Row gradients of the overlay: grad_rows[r, :] = sum over (t,h) with
 * slots[t,h] == r of the upstream gradient at (t,h), added from +0 in
 * ascending t*n_heads+h order -- the order in which the reference's
 * index_put_(accumulate=True) adds duplicates (serially on one CPU thread,
 * after a stable sort on CUDA), so the result is bit-identical to it and
 * deterministic.  Every row of grad_rows [R, dim] is written (zero where no
 * hit).  mode CONCAT_F32: grad float [n, n_heads, dim]; mode PAIRSUM_ADD_BF16:
 * grad bf16 [n, hpn*dim] (the term of (t,h) is grad[t, (h%hpn)*dim : +dim]).
 * workspace: device scratch of engram_backward_workspace_bytes(n, n_heads, R).
 */
ENGRAM_API int engram_backward(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram,
                    int32_t mode, const void* grad, int32_t dim, int64_t R, float* grad_rows,
                    void* workspace, int64_t workspace_bytes, void* stream);

/* Size of the library's own scratch array used by engram_backward_noalloc. */
#define ENGRAM_NOALLOC_SCRATCH_BYTES (12LL << 20)

/*
 * engram_backward without a workspace argument, for callers that cannot
 * allocate device memory when they need the row gradients: a host engine
 * that reserves all of its GPU memory up front and forbids allocation on the
 * serving/training path (the llama.cpp-style engines that consume .pleo
 * overlays work this way), or code that must not pay cudaMalloc's implicit
 * device-wide synchronisation in the middle of a step.  It has no counterpart
 * in the reference, which always lets torch allocate.
 *
 * The caller still passes every input and output; the scratch lives in one
 * file-scope device array of ENGRAM_NOALLOC_SCRATCH_BYTES (12 MiB) that every
 * GPU which loads the library keeps until the process exits.  Sizes whose
 * engram_backward_workspace_bytes(n, n_heads, R) exceeds that return
 * ENGRAM_ERR_WORKSPACE and launch nothing (about n*n_heads <= 500,000 entries
 * with R <= 500,000 rows fits).  The first call on a device looks up the
 * array's device address with that device current, so make that first call
 * before any stream capture.  The address is kept for the life of the
 * process: cudaDeviceReset on that device ends the context holding the array,
 * and this entry point must not be called on that device afterwards.  All
 * calls share the array: two calls whose
 * kernels overlap on the GPU (different streams, or different host threads on
 * one device) race and corrupt each other's results, so serialise them.
 * Nothing in the array needs to start at zero: each call writes every scratch
 * byte it later reads.  Results are bit-identical to engram_backward.
 */
ENGRAM_API int engram_backward_noalloc(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram,
                                       int32_t mode, const void* grad, int32_t dim, int64_t R, float* grad_rows,
                                       void* stream);

/*
 * One optimizer step over numel fp32 elements, in place on p, m, v:
 *   g  = g_in + reg_scale * (2*(p - p0))        (p0 NULL: g = g_in)
 *   m  = fma(1-beta1, g-m, m)                   (torch lerp)
 *   v  = v*beta2 + ((1-beta2)*g)*g
 *   p  = p + (-(lr/(1-beta1^step)) * m) / (sqrt(v)/sqrt(1-beta2^step) + eps)
 * reg_scale = float(mu) / max(sum(p0^2), 1e-12): the factor autograd applies
 * to the descent's regulariser (engraft/descend_corpus.py:935-937); step >= 1
 * is the step count after this update (torch.optim.Adam, no weight decay).
 */
ENGRAM_API int engram_adam_step(float* p, const float* g, float* m, float* v, const float* p0, int64_t numel,
                     int64_t step, double lr, double beta1, double beta2, double eps, float reg_scale,
                     void* stream);

/*
 * Data-parallel ranks over peer memory (no reference counterpart: the reference
 * is single-process).  The overlay rows are sharded by owner: rank o owns the
 * contiguous rows [o*(R/W) + min(o, R%W), +size_o), size_o = R/W + (o < R%W).
 * Each rank has a receive buffer [world, max size_o, dim] fp32 (16-byte aligned)
 * mapped into every process (e.g. torch symmetric memory).
 *
 * engram_backward_to_owners: engram_backward whose row of slot s is stored into
 * its owner's receive buffer, block `rank` (owner_bufs: device array [world] of
 * the receive buffers); the reduce-scatter's transfer happens inside the
 * reduction, as peer stores.
 *
 * engram_adam_owner_step: for the rows this rank owns, the sum of the world
 * blocks of its receive buffer in rank order, engram_adam_step's update (m, v,
 * p0 hold the owned rows only), and a store of the new rows into every rank's
 * rows_var (rows_ptrs: device array [world]); the all-gather's transfer
 * happens inside the update, as peer stores.
 *
 * Neither kernel waits on another GPU: every rank's backward must finish before
 * any owner step starts, and every owner step before any rank reads rows_var
 * (two barriers, e.g. tiny NCCL all-reduces on the stream).
 */
ENGRAM_API int engram_backward_to_owners(const int32_t* slots, int64_t n, int32_t n_heads, int32_t heads_per_ngram,
                                         int32_t mode, const void* grad, int32_t dim, int64_t R,
                                         const void* owner_bufs, int32_t world, int32_t rank, void* workspace,
                                         int64_t workspace_bytes, void* stream);
ENGRAM_API int engram_adam_owner_step(const float* recv, const void* rows_ptrs, int32_t world, int32_t rank,
                                      int64_t R, int32_t dim, float* m, float* v, const float* p0, int64_t step,
                                      double lr, double beta1, double beta2, double eps, float reg_scale,
                                      void* stream);

/* Scratch bytes engram_scan_hits needs for n positions. */
ENGRAM_API int64_t engram_scan_hits_workspace_bytes(int64_t n);

/*
 * Bulk hash + overlay hit scan over positions t0..t0+n-1 of `tokens` (no
 * segments; tokens before t0 are context), replacing damage.scan_hits +
 * ngram_rows (engraft/damage.py:68-104,168-224).  ov: the map of the overlay
 * rows sorted ascending (slot k = overlay_sorted[k]; ov->rows is not read);
 * dnorm: device float [R].  For every position whose rows include at least one
 * overlay row (and which is not the last one when exclude_last != 0), in
 * position order: pos_out (int64, pos_base + t), nhit_out (rows matched),
 * dmax_out / dsum_out (max and numpy-pairwise float32 sum over heads of
 * matched ? dnorm : 0).  *n_hits (device int64) = number listed; read_count
 * (device int64 [R]) += reads of each overlay row (all positions).  Outputs
 * are sized n.  Requires n_heads <= 16.
 */
ENGRAM_API int engram_scan_hits(const engram_table* t, const int32_t* tokens, int64_t t0, int64_t n, int64_t pos_base,
                                int32_t exclude_last, const engram_overlay* ov, const float* dnorm, int64_t* pos_out,
                                int32_t* nhit_out, float* dmax_out, float* dsum_out, int64_t* n_hits,
                                int64_t* read_count, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Row sets: sets of global table rows as device bitmaps (uint32 words, bit g%32
 * of word g/32 = row g).  They replace the Python sets of the row-set builders:
 * build_all_read_row_set (engraft/descend_corpus.py:1409-1430), build_rows_var
 * (engraft/replica/distill.py:401-457) and the union of sum_overlays
 * (engraft/replica/overlay_sum.py:36-112).  The caller zeroes a bitmap before
 * its first use.
 */
/* Words of a bitmap over n_rows rows. */
ENGRAM_API int64_t engram_rowset_words(int64_t n_rows);

/* Marks the rows read at positions: for each k < n, position positions[k]
 * (device int64; NULL: position k) of `tokens` (device int32 [n_tokens]),
 * hashed with its context as engram_hash does, all n_heads heads
 * (RowSet.from_position, engraft/lens.py:127-136).  Positions are clamped into
 * [0, n_tokens). */
ENGRAM_API int engram_rowset_mark(const engram_table* t, const int32_t* tokens, int64_t n_tokens,
                                  const int32_t* seg_start, const int64_t* positions, int64_t n, uint32_t* bitmap,
                                  void* stream);

/* Marks the given global ids (device int32 [n]); ids outside [0, n_rows) are skipped. */
ENGRAM_API int engram_rowset_mark_ids(const int32_t* ids, int64_t n, int64_t n_rows, uint32_t* bitmap, void* stream);

/* out = a | b (op 0), a & ~b (op 1) or a & b (op 2), word by word; out may alias a or b. */
ENGRAM_API int engram_rowset_combine(const uint32_t* a, const uint32_t* b, int64_t words, int32_t op, uint32_t* out,
                                     void* stream);

/* Scratch bytes engram_rowset_extract needs for a bitmap of `words` words. */
ENGRAM_API int64_t engram_rowset_workspace_bytes(int64_t words);

/* The members in ascending order: *count (device int64) = number of members;
 * ids_out (device int32 [capacity], nullable when capacity == 0) receives the
 * first min(count, capacity) of them.  The workspace then holds the bitmap's
 * word prefixes, which engram_rowset_index reads. */
ENGRAM_API int engram_rowset_extract(const uint32_t* bitmap, int64_t words, int32_t* ids_out, int64_t capacity,
                                     int64_t* count, void* workspace, int64_t workspace_bytes, void* stream);

/* index_out[k] = position of ids[k] in the ascending member list, or -1 when
 * ids[k] is not a member.  Needs the workspace of an engram_rowset_extract of
 * the same bitmap, run before on the same stream. */
ENGRAM_API int engram_rowset_index(const uint32_t* bitmap, int64_t words, const void* workspace,
                                   int64_t workspace_bytes, const int32_t* ids, int64_t n, int32_t* index_out,
                                   void* stream);

/* acc[index[k]] += data[k] - base[k] for k < n (rows of dim floats, fp32
 * subtract then add; index -1 skips a row): one .pleo file's deltas added into
 * the sum over the union of rows (engraft/replica/overlay_sum.py:80-96).
 * order (device int64 [n], nullable): the rows k sorted by index[k], stable;
 * with it, rows with the same target are added in ascending k (file order), as
 * np.add.at applies them, all in one launch.  Without it the targets must be
 * distinct. */
ENGRAM_API int engram_overlay_accumulate(float* acc, const int32_t* index, const int64_t* order, const float* data,
                                         const float* base, int64_t n, int32_t dim, void* stream);

/* Host self-test of the division magic: out[i] = x[i] % d using exactly the
 * device code path (host arrays).  Lets CPU-only tests check it. */
ENGRAM_API int engram_selftest_mod(const uint64_t* x, int64_t count, uint32_t d, uint64_t* out);

/* Number of CUDA kernels this library has launched in this process (all
 * entry points, all devices); lets callers verify that the CUDA path ran. */
ENGRAM_API int64_t engram_launch_count(void);

/* Library version (major*10000 + minor*100 + patch). */
ENGRAM_API int engram_version(void);

/*
 * The PLE block that consumes the gathered rows (engraft/replica/layers.py:
 * 565-626, ple_forward), after its two projections key = emb @ w_key.T
 * [T, hc*n] and value = emb @ w_value.T [T, n] (plain GEMMs, run by the
 * caller).  fp32 throughout; hc <= 8, n % 4 == 0; row strides in floats,
 * multiples of 4; arrays 16-byte aligned.
 * engram_ple_gate: per position t and stream j,
 *   s = <rmsnorm(key_j) * norm_key_j, rmsnorm(hidden_j) * norm_query_j> / sqrt(n),
 *   gate[t, j] = sigmoid(sign(s) * sqrt(max(|s|, 1e-6))), s_out (nullable) = s,
 *   normed[t, j, :] = rmsnorm(value * gate) * norm_conv_j,
 *   with rmsnorm(x) = x * rsqrt(mean(x^2) + eps) (layers.py:23-42).
 * engram_ple_conv: out[t, j, c] = hidden + value[t, c] * gate[t, j] +
 *   silu(sum_k conv_w[j*n + c, k] * x[t - (K-1-k)*dilation]), x = normed rows,
 *   or hist rows [hist_len, hc, n] before position 0, or 0 before the history
 *   (causal_depthwise_conv, layers.py:257-293).
 */
ENGRAM_API int engram_ple_gate(const float* key, int64_t key_stride, const float* value, int64_t value_stride,
                               const float* hidden, const float* norm_key, const float* norm_query,
                               const float* norm_conv, int64_t T, int32_t hc, int32_t n_embd, float eps,
                               float* gate, float* s_out, float* normed, void* stream);
ENGRAM_API int engram_ple_conv(const float* value, int64_t value_stride, const float* hidden, const float* gate,
                               const float* normed, const float* hist, int64_t hist_len, const float* conv_w,
                               int32_t K, int32_t dilation, int64_t T, int32_t hc, int32_t n_embd, float* out,
                               void* stream);

/*
 * Backward of the PLE block after its projections (the autograd of
 * engraft/replica/layers.py:565-626 that the descent's loss.backward() runs,
 * engraft/replica/seq.py:1457-1462), fp32.
 * engram_ple_gate_backward, per position t and stream j, from the forward's
 *   inputs (key = emb @ w_key.T before its norm, value, hidden, the three norm
 *   weights), its gate and s (engram_ple_gate's gate and s_out), the gradient
 *   of out (dout [T, hc, n]) and of normed (dnormed [T, hc, n], from
 *   engram_ple_conv_backward): dkey [T, hc*n] (row stride dkey_stride, the
 *   gradient of key), dvalue [T, n] (row stride dvalue_stride) and dhidden
 *   [T, hc, n] (the direct term of out plus the query norm's).  detach_value /
 *   detach_gate: the reference's flags (the value, or the gate, gets no
 *   gradient through gated = value * gate).  The projections' own backward,
 *   d_emb = dkey @ w_key + dvalue @ w_value, is a GEMM the caller runs.
 * engram_ple_conv_backward: dconv (device scratch [T, hc*n]) = dout * silu'(conv)
 *   with conv recomputed from normed and hist; then the transposed conv:
 *   dnormed [T, hc, n] and dhist [hist_len, hc, n] (nullable: not wanted),
 *   adding dtail [tail_len, hc, n] (nullable), the gradient of the new history
 *   tail (the last tail_len rows of [hist; normed]).
 * Agrees with torch's autograd of the reference to fp32 rounding.
 */
ENGRAM_API int engram_ple_gate_backward(const float* key, int64_t key_stride, const float* value, int64_t value_stride,
                                        const float* hidden, const float* norm_key, const float* norm_query,
                                        const float* norm_conv, const float* gate, const float* s, const float* dout,
                                        const float* dnormed, int64_t T, int32_t hc, int32_t n_embd, float eps,
                                        int32_t detach_value, int32_t detach_gate, float* dkey, int64_t dkey_stride,
                                        float* dvalue, int64_t dvalue_stride, float* dhidden, void* stream);
ENGRAM_API int engram_ple_conv_backward(const float* normed, const float* hist, int64_t hist_len, const float* conv_w,
                                        int32_t K, int32_t dilation, int64_t T, int32_t hc, int32_t n_embd,
                                        const float* dout, const float* dtail, int64_t tail_len, float* dconv,
                                        float* dnormed, float* dhist, void* stream);

/*
 * C[M, N] (row stride ldc floats) = sum over p < n_terms (1..3) of
 * A_p[M, K] @ B_p[N, K]^T on the tensor cores (tcgen05.mma kind::tf32, operands
 * loaded by TMA, fp32 accumulation in tensor memory): a and b are HOST arrays
 * of n_terms device pointers to row-major fp32 matrices (row strides lda, ldb
 * floats; K, lda, ldb multiples of 4; 16-byte aligned), each element read as
 * TF32.  With the terms (A_lo, B_hi), (A_hi, B_lo), (A_hi, B_hi) of the split
 * x = hi + lo (hi: x with its low 13 mantissa bits cleared) the result is the
 * 3xTF32 product, fp32-level accurate: the PLE block's projections
 * (engraft/replica/layers.py:587,593, key = emb @ w_key.T, value = emb @
 * w_value.T) and their backward.  err (device int32, nullable) counts
 * barrier waits that gave up (a bounded spin; 0 in any correct run).
 */
ENGRAM_API int engram_gemm_tf32(int32_t n_terms, const float* const* a, const float* const* b, int64_t M, int64_t N,
                                int64_t K, int64_t lda, int64_t ldb, float* c, int64_t ldc, int32_t* err,
                                void* stream);
/*
 * The same 3xTF32 product from the split operands in one pass: C = A_lo B_hi^T
 * + A_hi B_lo^T + A_hi B_hi^T with A_hi, A_lo sharing row stride lda and B_hi,
 * B_lo sharing ldb.  Each K slice of the four operands is loaded once and the
 * three MMAs are issued from it (a third less operand traffic than
 * engram_gemm_tf32 with three terms).  Same shape rules and err.
 */
ENGRAM_API int engram_gemm_3xtf32(const float* a_hi, const float* a_lo, const float* b_hi, const float* b_lo,
                                  int64_t M, int64_t N, int64_t K, int64_t lda, int64_t ldb, float* c, int64_t ldc,
                                  int32_t* err, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* ENGRAM_B200_H */

/* stade_emit.h -- the .cu emitter: STADE-generated Julia sweep in, CUDA out.
 *
 * Replaces stade_cuda_file (src/STADE.jl:12062-12111 cgen_emit, with the
 * loop -> kernel decisions of cgen_body, src/STADE.jl:10409-10640) for sweeps
 * beyond the hand-written ones: it reads the text of a generated `<k>_b.jl`
 * (or `_d.jl`, `_hv.jl`) holding `<k>_b(...)` and `initstacks_<k>_b(...)`,
 * and writes one CUDA source that defines
 *
 *   int     stade_<k>_b(<generated argument order>, void* stream);
 *   int64_t stade_initstacks_<k>_b(<int arguments>, int64_t* sizes, int* dtypes,
 *                                  void* const* fill);
 *
 * Arguments keep the generated order. Float arrays are T* (T = double, or
 * float with precision 32, as cgen_convert_precision), integer arrays and
 * stacks int64_t*, integer scalars int64_t by value, float scalars by value
 * unless the sweep returns them (their adjoints), in which case they are T*
 * host pointers updated in place (the generated code returns them by value,
 * emit_return_scalars src/STADE.jl:2072). stade_initstacks_<k>_b runs
 * initstacks_<k>_b's statements on the host (the closed-form tape layout of
 * agen_indexed_layout, src/STADE.jl:4917, or the Tier-B sizing loop of
 * agen_tier_b_block_stmts, src/STADE.jl:5338-5380) and returns the number
 * of items it returns; per item i, sizes[i] and dtypes[i]:
 *   0 / 1 / 2  a stack (Float64 / Float32 / Int64) of sizes[i] elements the
 *              caller allocates and zero-fills (the library never allocates);
 *   3          an integer (a running total, a length): its value in sizes[i];
 *   4 / 5      a table initstacks fills (Int64 / the sweep's float type) of
 *              sizes[i] elements: with fill non-NULL and fill[i] a host buffer
 *              of that size, its contents are written there.
 * An argument initstacks reads only through length(a) is passed as that
 * length (the manifest lists these as "length_args"). It returns -1 when a
 * table write falls outside the table.
 *
 * An array the sweep allocates at its top level in Julia (an HVP sweep's
 * tangent of a tape, `du_stack_d = Vector{Float64}(undef, length(du_stack))`)
 * becomes a trailing argument of stade_<k>, after the generated ones; the
 * caller allocates it. Its size comes from
 *
 *   int64_t stade_<k>_locals(<integer arguments>, <lengths of the arrays the
 *                            sizes read through length()>, int64_t* sizes,
 *                            int* dtypes);
 *
 * (dtype 0 / 1 / 2 as for stacks; the manifest's "locals" names them). An
 * HVP sweep <k>_hv takes its stacks from initstacks_<k>_b.
 *
 * Calls of one emitted sweep share its file-scope device boxes (the boxed
 * scalars and the returned scalar adjoints live in one __device__ array per
 * emitted library): order the calls of one sweep on one stream, or put events
 * between streams. Two calls that overlap on the GPU race on the boxes, and
 * one can read back the other's returned scalars. Different emitted sweeps
 * have separate boxes.
 *
 * The manifest (JSON) lists the arguments with their kinds, the stacks, the
 * returned scalars and one record per loop: parallel kernel (thread per
 * iteration, with the arrays and scalars it updates by atomics and the
 * scalars private to an iteration) or sequential (one thread), with the
 * reason.
 */
#ifndef STADE_EMIT_H
#define STADE_EMIT_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Emits CUDA source for function `function` (NULL: the first function whose
 * name does not start with "initstacks_" and that has a matching
 * initstacks_ function, else the first function) of the Julia text `source`.
 * precision: 64 or 32. dims: leading dimensions of multi-dimensional arrays,
 * "a=i_m,i_n;b=3,n_c" (NULL or "": inferred from the loops that index them).
 * Writes NUL-terminated text into cu / manifest when their capacity allows;
 * *cu_len and *manifest_len receive the lengths needed (without the NUL).
 * Returns 0, or 1 with stade_emit_last_error() describing the failure. */
int stade_emit_cuda(const char* source, const char* function, int precision, const char* dims,
                    char* cu, size_t cu_cap, size_t* cu_len, char* manifest,
                    size_t manifest_cap, size_t* manifest_len);

const char* stade_emit_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* STADE_EMIT_H */

/* Host shim that compiles the reference's NF4 compute shaders
 * (src/alelyon_compute_kit/_kit/kernels/nf4_decode.comp and nf4_gemv.comp,
 * GLSL 450) as C++. TEST INFRASTRUCTURE ONLY: the results under oracle/_ref/
 * are checkers for the numpy restatement in nf4_oracle.py; nothing in the
 * product loads them.
 *
 * oracle/Makefile feeds each shader's text to g++ unchanged except that its
 * `#version` and `#extension` lines (directives C++ does not have) are
 * blanked, so diagnostics keep the shader's line numbers; the variant macros
 * (STORAGE for the decode, ELEM_F16 and ROWS_CAP for the product) come from
 * -D flags.
 *
 * How each GLSL construct maps (as in vq4_shim.h, with typed bindings):
 *   - `layout(...)`, `readonly`, `writeonly`, `precise` vanish; `in;` is an
 *     empty declaration. -ffp-contract=off and -fsingle-precision-constant
 *     on x86-64 SSE make every FP32 operation round once, in source order.
 *   - A storage block member `T name[]` is a macro for `(*g_name)`, a
 *     bounds-checked array of the host's choosing (an index past it reads 0,
 *     drops the write and marks the call bad).
 *   - `uniform P {...} p;` is a plain struct (the push constants).
 *   - `uvec4` is four u32 words with indexing; `findMSB` is the bit scan.
 *   - nf4_decode.comp has no barrier: its invocations run one at a time.
 *   - nf4_gemv.comp's workgroups share `partial[][]` and meet at
 *     `barrier()`: its 64 invocations run as 64 host threads that start each
 *     workgroup together, meet at every `barrier()` (a std::barrier) and
 *     finish it together, workgroups one after another.
 */
#include <barrier>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

typedef uint32_t uint;

template <typename T>
struct GlslArr {
    T *data;
    uint64_t count;
    int bad;
    T &operator[](uint64_t i) {
        static thread_local T sink;
        if (i >= count) { bad = 1; sink = T(); return sink; }
        return data[i];
    }
};

struct uvec4 {
    uint32_t w[4];
    uint32_t &operator[](uint32_t i) { return w[i]; }
    const uint32_t &operator[](uint32_t i) const { return w[i]; }
};

struct GlslUvec3 { uint32_t x, y, z; };

static thread_local GlslUvec3 gl_WorkGroupID, gl_NumWorkGroups, gl_LocalInvocationID, gl_GlobalInvocationID;

static inline float uintBitsToFloat(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
static inline uint32_t floatBitsToUint(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline uint32_t min(uint32_t x, uint32_t y) { return x < y ? x : y; }
static inline int findMSB(uint32_t v) { return v ? 31 - __builtin_clz(v) : -1; }

static std::barrier<> *g_sync;
static inline void barrier() { g_sync->arrive_and_wait(); }

/* nf4_decode.comp's bindings */
static GlslArr<uint32_t> *g_packed_words, *g_absmax_q_words, *g_start_words, *g_id_words;
static GlslArr<float> *g_absmax2_values, *g_table_values, *g_offset_values;
#if defined(STORAGE) && STORAGE != 0
static GlslArr<uint16_t> *g_output_values;
#else
static GlslArr<float> *g_output_values;
#endif
/* nf4_gemv.comp's bindings (packed_words is shared with the decode) */
static GlslArr<uvec4> *g_a;
static GlslArr<float> *g_c, *g_absmax2, *g_tables, *g_offsets;
static GlslArr<uint32_t> *g_absmax_q, *g_starts, *g_groups;

#define layout(...)
#define in
#define readonly
#define writeonly
#define buffer struct
#define uniform struct
#define precise
#define shared static
#define packed_words (*g_packed_words)
#define absmax_q_words (*g_absmax_q_words)
#define absmax2_values (*g_absmax2_values)
#define table_values (*g_table_values)
#define start_words (*g_start_words)
#define offset_values (*g_offset_values)
#define id_words (*g_id_words)
#define output_values (*g_output_values)
#define a (*g_a)
#define c (*g_c)
#define absmax_q (*g_absmax_q)
#define absmax2 (*g_absmax2)
#define tables (*g_tables)
#define starts (*g_starts)
#define offsets (*g_offsets)
#define groups (*g_groups)
#define main nf4_glsl_main

static void nf4_glsl_main();

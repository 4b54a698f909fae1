/* Host shim that compiles the reference's vq4 compute shader source
 * (src/alelyon_compute_kit/_kit/kernels/vq4.comp, GLSL 450) as C++.
 * TEST INFRASTRUCTURE ONLY: the result, oracle/_ref/libvq4_ref.so, is a
 * checker for the numpy restatements in vq_oracle.py; nothing in the product
 * loads it.
 *
 * The shader's arithmetic is plain 32-bit integer and FP32 work, so it needs
 * no graphics stack. oracle/Makefile feeds the unchanged shader text to g++
 * with this header force-included; only its first line (`#version 450`,
 * which C++ has no directive for) is blanked on the way in, so line numbers
 * in diagnostics match the shader file.
 *
 * How each GLSL construct maps:
 *   - `layout(...)` qualifiers vanish; `in;` becomes an empty declaration.
 *   - A storage block `buffer In0 { uint b0[]; };` becomes a struct whose
 *     member is a pointer-to-array; the name `b0` is a macro for `(*g_b0)`,
 *     so the shader's `b0[i]` and `b0.length()` reach the global binding
 *     object `g_b0`, a bounds-checked u32 array of the host's choosing.
 *   - `uniform Push {...} p;` becomes a plain struct variable (the plan).
 *   - `precise` vanishes. The build uses -ffp-contract=off (no fused
 *     multiply-add) and -fsingle-precision-constant (a literal such as 1.0 is
 *     an FP32 constant, as in GLSL), on x86-64 SSE arithmetic (no excess
 *     precision), so every FP32 operation rounds once, in source order.
 *     Division and sqrt are IEEE correctly rounded here.
 *   - `atomicOr` is a plain OR: invocations run one at a time.
 *   - `main` is renamed and called once per invocation by vq4_ref_run(),
 *     which walks the same 2-D grid of 64-wide workgroups the reference's
 *     planner records (x = min(groups, 65535), y = ceil(groups / x)).
 */
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

typedef uint32_t uint;

struct GlslBinding {
    uint32_t *data;
    uint32_t count;
    int bad;
    uint32_t &operator[](uint32_t i) {
        static uint32_t sink;
        if (i >= count) { bad = 1; sink = 0; return sink; }
        return data[i];
    }
    int length() const { return (int)count; }
};

struct GlslUvec3 { uint32_t x, y, z; };

static GlslBinding *g_b0, *g_b1, *g_b2, *g_b3, *g_dst, *g_status;
static GlslUvec3 gl_WorkGroupID, gl_NumWorkGroups, gl_LocalInvocationID;

static inline float uintBitsToFloat(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
static inline uint32_t floatBitsToUint(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline void atomicOr(uint32_t &word, uint32_t bits) { word |= bits; }
static inline uint32_t min(uint32_t a, uint32_t b) { return a < b ? a : b; }
using std::isinf;
using std::isnan;
using std::sqrt;

#define layout(...)
#define in
#define readonly
#define writeonly
#define buffer struct
#define uniform struct
#define precise
#define b0 (*g_b0)
#define b1 (*g_b1)
#define b2 (*g_b2)
#define b3 (*g_b3)
#define dst (*g_dst)
#define status (*g_status)
#define main vq4_glsl_main

static void vq4_glsl_main();
static void vq4_set_plan(const uint32_t *plan);

/* Runs one dispatch of the shader over host arrays.
 * plan: the 8 u32 push constants [op, m, n, k, group, entries, flags, reserved].
 * bN / out / status: the six bindings, with their lengths in u32 words.
 * groups: workgroups to launch (the reference records ceil(invocations / 64)).
 * Returns 0, or 1 if the shader indexed past a binding (a shim-level check the
 * GPU does not make; the layout checks in the shader are still its own). */
extern "C" int vq4_ref_run(const uint32_t *plan,
                           uint32_t *in0, uint32_t n0, uint32_t *in1, uint32_t n1,
                           uint32_t *in2, uint32_t n2, uint32_t *in3, uint32_t n3,
                           uint32_t *out, uint32_t nout, uint32_t *stat, uint32_t nstat,
                           uint32_t groups) {
    GlslBinding bind[6] = {{in0, n0, 0}, {in1, n1, 0}, {in2, n2, 0},
                           {in3, n3, 0}, {out, nout, 0}, {stat, nstat, 0}};
    g_b0 = &bind[0]; g_b1 = &bind[1]; g_b2 = &bind[2]; g_b3 = &bind[3];
    g_dst = &bind[4]; g_status = &bind[5];
    vq4_set_plan(plan);
    uint32_t gx = groups < 65535u ? groups : 65535u;
    if (gx == 0) gx = 1;
    uint32_t gy = (groups + gx - 1) / gx;
    gl_NumWorkGroups.x = gx; gl_NumWorkGroups.y = gy; gl_NumWorkGroups.z = 1;
    gl_WorkGroupID.z = 0; gl_LocalInvocationID.y = 0; gl_LocalInvocationID.z = 0;
    for (uint32_t y = 0; y < gy; ++y)
        for (uint32_t x = 0; x < gx; ++x)
            for (uint32_t t = 0; t < 64u; ++t) {
                gl_WorkGroupID.x = x; gl_WorkGroupID.y = y; gl_LocalInvocationID.x = t;
                vq4_glsl_main();
            }
    int bad = 0;
    for (auto &b : bind) bad |= b.bad;
    return bad;
}

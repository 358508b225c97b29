/* ref_rtti_stub.c -- link helper for oracle/_ref/libmlxref.so (test infrastructure).
 *
 * MLX's core library, which defines mlx::core::Primitive and therefore emits
 * its typeinfo object, is not linked into the reference-kernel library. Inline
 * RTTI of derived primitives that survives in ref_mlx_cpu.cpp still names that
 * base typeinfo, so the loader wants the symbol. Nothing on the two called
 * paths (quantized matmul, quantize) uses RTTI; a hidden zeroed object of
 * typeinfo size satisfies the loader. Written in C so the mangled name can be
 * defined without clashing with the C++ compiler's own declaration. */
__attribute__((visibility("hidden"), aligned(16)))
char _ZTIN3mlx4core9PrimitiveE[16] = {0};

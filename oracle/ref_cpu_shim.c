/* ref_cpu_shim.c — TEST INFRASTRUCTURE ONLY. Exposes the reference's own CPU attention.
 *
 * The reference's attention() in cpu/forward_cpu.c:83-116 is `static`, so this translation unit pulls
 * the unmodified reference source in with #include (the include path points at the reference tree;
 * nothing is copied into this repository) and exports one C entry point around it. oracle/Makefile
 * builds it into oracle/_ref/libref_cpu.so with the reference's own flag set (gcc -O2 -fopenmp).
 *
 * Used by tests (to pin oracle/attn_oracle.c and to make tests/golden/) and by bench.py's reference
 * arm / cpu_baseline, which time this exact code on the host cores. The include also exports the
 * reference's whole fp32 forward, gpt2_forward_cpu (cpu/forward_cpu.c:118), unchanged: the decode
 * step tests use it as the CPU oracle of the model around the attention.
 */
#include "forward_cpu.c"

/* att[T, 768] = causal attention of qkv[T, 2304] (fp32, GPT-2-124M shapes, 1 <= T <= 1024). */
int ref_cpu_attention(float *att, const float *qkv, int T) {
    if (T < 1 || T > GPT2_N_CTX) return -1;
    attention(att, qkv, T);
    return 0;
}

int ref_cpu_n_ctx(void) { return GPT2_N_CTX; }

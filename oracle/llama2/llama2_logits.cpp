// llama2_logits.cpp — TEST INFRASTRUCTURE: a driver around akili-bench's
// unchanged benchmarks/llama2/llama.cpp, compiled in place with TESTING
// defined (which leaves out its command-line main, llama2/llama.cpp:913-1011).
// It runs the reference forward pass (llama2/llama.cpp:246-407) on a fixed
// token sequence, one position at a time, and writes every position's logits
// as raw fp32 to a file, so that runs with the CPU matmul (use_vortex = 0,
// llama2/llama.cpp:235-243) and with an offload library (use_vortex = 1)
// can be compared position by position.
//
//   llama2_logits <checkpoint> <use_vortex> <out.bin> <tok_0> ... <tok_T-1>
#define TESTING
#include "llama.cpp"

int main(int argc, char* argv[]) {
  if (argc < 5) {
    fprintf(stderr, "usage: %s <checkpoint> <use_vortex> <out.bin> <tok_0> ... <tok_T-1>\n", argv[0]);
    return 2;
  }
  use_vortex = atoi(argv[2]) != 0;
  if (use_vortex) vx_init();
  Transformer transformer;
  build_transformer(&transformer, argv[1]);
  const int T = argc - 4;
  if (T > transformer.config.seq_len) {
    fprintf(stderr, "%d tokens exceed seq_len %d\n", T, transformer.config.seq_len);
    return 2;
  }
  FILE* out = fopen(argv[3], "wb");
  if (!out) return 2;
  for (int pos = 0; pos < T; ++pos) {
    const int tok = atoi(argv[4 + pos]);
    if (tok < 0 || tok >= transformer.config.vocab_size) return 2;
    float* logits = forward(&transformer, tok, pos);
    fwrite(logits, sizeof(float), transformer.config.vocab_size, out);
  }
  fclose(out);
  free_transformer(&transformer);
  if (use_vortex) matmul_cleanup();
  return 0;
}

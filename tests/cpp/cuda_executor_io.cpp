// Drives runtime::gpu::cuda_softmax / cuda_attention (include/cuda_executor.h)
// from binary files.  argv: mode in.bin out.bin
//   softmax:   in = u64 rows, u64 cols, rows*cols fp32
//   attention: in = u64 seq, u64 dim, Q, K, V (seq*dim fp32 each)
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "cuda_executor.h"

int main(int argc, char **argv) {
    if (argc < 4) return 1;
    FILE *f = fopen(argv[2], "rb");
    if (!f) return 2;
    uint64_t a = 0, b = 0;
    if (fread(&a, 8, 1, f) != 1 || fread(&b, 8, 1, f) != 1) return 3;
    const bool attn = strcmp(argv[1], "attention") == 0;
    const size_t n = (size_t)a * b;
    std::vector<float> x(n * (attn ? 3 : 1)), y(n);
    if (fread(x.data(), 4, x.size(), f) != x.size()) return 4;
    fclose(f);
    if (!runtime::gpu::cuda_available() || !runtime::gpu::cuda_init()) return 5;
    const bool ok = attn ? runtime::gpu::cuda_attention(x.data(), x.data() + n, x.data() + 2 * n, y.data(), a, b)
                         : runtime::gpu::cuda_softmax(x.data(), y.data(), a, b);
    if (!ok) return 6;
    FILE *o = fopen(argv[3], "wb");
    fwrite(y.data(), 4, y.size(), o);
    fclose(o);
    return 0;
}

// Runs KvAttentionBackend (include/kv_backend.h) over `steps` decode steps:
// argv: config.txt inputs.bin outputs.bin steps.  inputs.bin holds, for
// every step and layer, one fp32 tensor {B, q_heads + 2*kv_heads, 128};
// the outputs {B, q_heads, 128} are written in the same order.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "kv_backend.h"

int main(int argc, char **argv) {
    if (argc < 5) return 1;
    KvAttentionBackend be;
    if (!be.load(argv[1])) return 2;
    const runtime::ModelMetadata md = be.metadata();
    if (md.name != "kvx-paged-attention" || md.num_layers <= 0) return 3;
    FILE *in = fopen(argv[2], "rb");
    FILE *out = fopen(argv[3], "wb");
    if (!in || !out) return 4;
    const int steps = atoi(argv[4]);
    size_t row = 0;
    for (int s = 0; s < steps; ++s)
        for (int l = 0; l < md.num_layers; ++l) {
            runtime::Tensor x;
            uint64_t n = 0;
            if (fread(&n, 8, 1, in) != 1) return 5;
            x.data.resize(n);
            if (fread(x.data.data(), 4, n, in) != n) return 6;
            runtime::Tensor y = be.runLayer(l, x);
            if (y.data.empty()) return 7;
            row = y.data.size();
            fwrite(y.data.data(), 4, y.data.size(), out);
        }
    fclose(in);
    fclose(out);
    printf("ok %zu\n", row);
    return 0;
}

// Drives KVCompressionEngine (include/KVCompressionEngine.h) over the cases
// in argv[1]: records {int32 type, uint64 count, float[count]}.  For each it
// writes to argv[2]: float ratio, float stats[4], int32 stats.type, uint64
// compressed bytes, the compressed bytes, then the decompressed floats.
#include <cstdio>
#include <vector>

#include "KVCompressionEngine.h"

int main(int argc, char **argv) {
    if (argc < 3) return 1;
    FILE *in = fopen(argv[1], "rb");
    FILE *out = fopen(argv[2], "wb");
    if (!in || !out) return 2;
    KVCompressionEngine eng;
    int n_cases = 0;
    for (;;) {
        int32_t type = 0;
        uint64_t count = 0;
        if (fread(&type, 4, 1, in) != 1) break;
        if (fread(&count, 8, 1, in) != 1) return 3;
        std::vector<float> x(count);
        if (fread(x.data(), 4, count, in) != count) return 4;
        eng.setCompressionType(static_cast<CompressionType>(type));
        if (eng.getStrategy() != static_cast<CompressionType>(type)) return 5;
        const uint64_t nbytes = eng.getCompressedSize(static_cast<CompressionType>(type), count);
        std::vector<unsigned char> c(nbytes);
        QuantizationStats st{};
        const float ratio = eng.compress(x.data(), c.data(), count, st);
        std::vector<float> back(count);
        eng.decompress(c.data(), back.data(), count, st);
        const float s4[4] = {st.minVal, st.maxVal, st.scale, st.zeroPoint};
        const int32_t t = static_cast<int32_t>(st.type);
        fwrite(&ratio, 4, 1, out);
        fwrite(s4, 4, 4, out);
        fwrite(&t, 4, 1, out);
        fwrite(&nbytes, 8, 1, out);
        fwrite(c.data(), 1, nbytes, out);
        fwrite(back.data(), 4, count, out);
        ++n_cases;
    }
    fclose(in);
    fclose(out);
    printf("ok %d\n", n_cases);
    return 0;
}

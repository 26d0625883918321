// Writes one page through KVManager::save_page; the caller compares the file
// with the reference's bytes.  argv: dir, id, key.bin, value.bin (raw fp32).
#include <cstdio>
#include <fstream>
#include <iterator>
#include <vector>

#include "kv_cache.h"

static std::vector<float> read_floats(const char *path) {
    std::ifstream in(path, std::ios::binary);
    std::vector<char> b((std::istreambuf_iterator<char>(in)), std::istreambuf_iterator<char>());
    std::vector<float> f(b.size() / 4);
    if (!f.empty()) std::copy(b.begin(), b.begin() + f.size() * 4, reinterpret_cast<char *>(f.data()));
    return f;
}

int main(int argc, char **argv) {
    if (argc < 5) return 1;
    KVManager m(4, argv[1]);
    KVPage p;
    p.id = atoi(argv[2]);
    p.key = read_floats(argv[3]);
    p.value = read_floats(argv[4]);
    m.save_page(p);
    m.evict_page(p.id);
    KVPage back = m.load_page(p.id);  // reload through the fp16 disk tier
    FILE *f = fopen((std::string(argv[1]) + "/back.bin").c_str(), "wb");
    fwrite(back.key.data(), 4, back.key.size(), f);
    fwrite(back.value.data(), 4, back.value.size(), f);
    fclose(f);
    return 0;
}

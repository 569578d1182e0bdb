// Host-side dump of the interleaved sequence parts that a partitioned context
// uses (vibevoice.cpp_b200/csrc/common.cuh: zz_part, zz_count, zz_local_row,
// the same inline functions the engine's host code and the kernels call).
// For every position p < n it writes the int32 record
//   zz_part(p), zz_count(0, p), zz_count(1, p),
//   then for part 0 and part 1 the row (pos p, cidx p, kvlen p + 1) as that
//   part sees it: local pos, local cidx, local kvlen
// (9 ints per position).  Built and run by tests/test_partition_cpu.py,
// which checks it against vibevoice.cpp_b200/partition.py.
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "common.cuh"

using namespace vvq2;

int main(int argc, char** argv) {
    if (argc != 3) return 2;
    const int n = std::atoi(argv[1]);
    std::vector<int> out;
    out.reserve((size_t)n * 9);
    for (int p = 0; p < n; ++p) {
        out.push_back(zz_part(p));
        out.push_back(zz_count(0, p));
        out.push_back(zz_count(1, p));
        RowMeta r;
        r.seq = 0;
        r.pos = p;
        r.cidx = p;
        r.kvlen = p + 1;
        for (int part = 0; part < 2; ++part) {
            const RowMeta l = zz_local_row(r, part);
            out.push_back(l.pos);
            out.push_back(l.cidx);
            out.push_back(l.kvlen);
        }
    }
    FILE* f = std::fopen(argv[2], "wb");
    if (!f) return 3;
    const size_t w = std::fwrite(out.data(), sizeof(int), out.size(), f);
    std::fclose(f);
    return w == out.size() ? 0 : 4;
}

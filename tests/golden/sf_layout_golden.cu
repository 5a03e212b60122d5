// Golden-vector generator for the NVFP4 scale-factor layout.
//
// The reference builds its SFA/SFB index tables from CUTLASS's
// Sm1xxBlkScaledConfig<16>::tile_atom_to_shape_SF{A,B}
// (src/cutlass_gemm/csrc/gemm/nvfp4.cu:122-147): tile_to_shape of the K-major
// atom ((32,4),(16,4)):((16,4),(0,1)) over (rows, K) with Step<_2,_1>. This
// program evaluates that exact CuTe layout (CUTLASS headers, host only) and
// prints, per shape, the byte offset of every natural scale (row, block) and
// the filter_zeros size, as JSON on stdout. make_golden.py commits the result.
#include <cstdio>
#include <cute/layout.hpp>

using namespace cute;

using SfKMajorAtom = Layout<Shape<Shape<_32, _4>, Shape<_16, _4>>, Stride<Stride<_16, _4>, Stride<_0, _1>>>;

int main() {
  const int shapes[][2] = {{1, 16}, {130, 64}, {160, 256}, {136, 288}, {257, 96}, {384, 1024}};
  std::printf("[");
  for (int s = 0; s < 6; ++s) {
    const int rows = shapes[s][0], k = shapes[s][1];
    auto layout = tile_to_shape(SfKMajorAtom{}, make_shape(rows, k), Step<_2, _1>{});
    const long total = static_cast<long>(cute::size(filter_zeros(layout)));
    std::printf("%s{\"rows\": %d, \"k\": %d, \"size\": %ld, \"offsets\": [", s ? ", " : "", rows, k, total);
    for (int r = 0; r < rows; ++r) {
      for (int b = 0; b < k / 16; ++b) {
        std::printf("%s%ld", (r || b) ? ", " : "", static_cast<long>(layout(make_coord(r, b * 16))));
      }
    }
    std::printf("]}");
  }
  std::printf("]\n");
  return 0;
}

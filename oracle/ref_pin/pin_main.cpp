// Pin driver: runs the reference's own RoPE table builders and Philox RNG
// (compiled from the reference sources, see Makefile) and writes their
// outputs as raw little-endian float32 blocks to stdout, in this order:
//   1. PhiloxRNG(42).randn(4096)            (counter offset 0)
//   2. PhiloxRNG(42).randn(4096) again      (counter offset 1)
//   3. PhiloxRNG(0x1234567890ABCDEF).randn(1000)
//   4. get_freqs(16), get_freqs(24)         (theta 10000)
//   5. compute_text_rope(7, 128)
//   6. compute_visual_rope(3,4,5, {32,48,48}, {1,1,1})
//   7. compute_visual_rope(3,4,5, {32,48,48}, {1,2,2})
//   8. compute_visual_rope(5,16,16, {32,48,48}, {1,2,2}) rows 0,1,17,255,256,1279
//   9. compute_visual_rope(31,32,32,{32,48,48}, {1,1,1}) rows 0, 1023, 1024, 31743
//  10. compute_visual_rope(3,4,5, {16,24,24}, {1,2,2})   (the lite video model's head_dim 64)
#include <cstdio>
#include <vector>
#include "rng.hpp"
#include "rope.hpp"

static void put(const std::vector<float>& v) { fwrite(v.data(), sizeof(float), v.size(), stdout); }

int main() {
    PhiloxRNG a(42);
    put(a.randn(4096));
    put(a.randn(4096));
    PhiloxRNG b(0x1234567890ABCDEFull);
    put(b.randn(1000));
    put(rope::get_freqs(16));
    put(rope::get_freqs(24));
    put(rope::compute_text_rope(7, 128));
    put(rope::compute_visual_rope(3, 4, 5, {32, 48, 48}, {1.0f, 1.0f, 1.0f}));
    put(rope::compute_visual_rope(3, 4, 5, {32, 48, 48}, {1.0f, 2.0f, 2.0f}));
    {
        auto t = rope::compute_visual_rope(5, 16, 16, {32, 48, 48}, {1.0f, 2.0f, 2.0f});
        for (int r : {0, 1, 17, 255, 256, 1279}) put(std::vector<float>(t.begin() + r * 128, t.begin() + (r + 1) * 128));
    }
    {
        auto t = rope::compute_visual_rope(31, 32, 32, {32, 48, 48}, {1.0f, 1.0f, 1.0f});
        for (int r : {0, 1023, 1024, 31743}) put(std::vector<float>(t.begin() + (size_t)r * 128, t.begin() + ((size_t)r + 1) * 128));
    }
    put(rope::compute_visual_rope(3, 4, 5, {16, 24, 24}, {1.0f, 2.0f, 2.0f}));
    return 0;
}

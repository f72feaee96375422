// Synthetic GGUF checkpoint writer (host only).
#pragma once
#include <cstdint>
#include <string>

namespace qdec {
// Write the checkpoint `preset` ("tiny", "27b", "27b-L<n>") seeded with `seed` to `path` using `threads`
// threads (0 = all).  Throws std::exception on failure.
void synth_gguf(const std::string &path, const std::string &preset, uint64_t seed, int threads);
}  // namespace qdec

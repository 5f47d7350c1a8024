// The library's host-side parts that need no GPU, driven on the CPU: the fork-join pool that lays
// out a run's lines (every part of every job exactly once, jobs back to back, any part count, a
// pool without threads) and the stager's streaming copy (every length and alignment, nothing
// outside the destination range written).  Prints "ok" and exits 0, or names the first failure.
#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <vector>

#include "host_pool.h"
#include "stager.h"

static int check_pool(crec::HostPool& pool, int jobs) {
  for (int rep = 0; rep < jobs; ++rep) {
    const int parts = (rep * 37) % 211;
    std::vector<std::atomic<int>> hits(static_cast<size_t>(parts));
    for (auto& h : hits) h.store(0);
    pool.run(parts, [&](int i) { hits[static_cast<size_t>(i)].fetch_add(1); });
    for (int i = 0; i < parts; ++i)
      if (hits[static_cast<size_t>(i)].load() != 1) {
        std::printf("pool of %d threads, job %d: part %d of %d ran %d times\n", pool.threads(), rep, i, parts,
                    hits[static_cast<size_t>(i)].load());
        return 1;
      }
  }
  return 0;
}

int main() {
  {
    crec::HostPool pool(7);
    if (check_pool(pool, 3000)) return 1;
  }
  {
    crec::HostPool solo(0);
    if (solo.threads() != 1 || check_pool(solo, 50)) return 1;
  }
  std::vector<uint8_t> src(512), dst(640);
  for (size_t i = 0; i < src.size(); ++i) src[i] = static_cast<uint8_t>(i * 131 + 7);
  for (int sa = 0; sa < 32; ++sa)
    for (int da = 0; da < 32; ++da)
      for (int n = 0; n <= 300; n += (n < 80 ? 1 : 7)) {
        std::memset(dst.data(), 0xA5, dst.size());
        crec::copy_streaming(dst.data() + 64 + da, src.data() + sa, static_cast<size_t>(n));
        crec::stores_visible();
        for (int i = 0; i < static_cast<int>(dst.size()); ++i) {
          const int k = i - 64 - da;
          const uint8_t want = k >= 0 && k < n ? src[static_cast<size_t>(sa + k)] : 0xA5;
          if (dst[static_cast<size_t>(i)] != want) {
            std::printf("copy_streaming: source offset %d, destination offset %d, %d bytes: byte %d\n", sa, da, n, i);
            return 1;
          }
        }
      }
  std::printf("ok\n");
  return 0;
}

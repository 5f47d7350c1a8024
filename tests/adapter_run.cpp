// Test driver: INTEGRATION.md's adapter (carbon::B200RecModels, extracted from the document at
// build time into adapter.inc) run through the reference's carbon::PipelineModels interface, the
// way carbon::Pipeline's recognize stage drives its device (carbon/src/pipeline.cpp:560-640): page
// groups given by set_pages, the next group by prefetch_pages while the current one is read,
// recognize a bucket width at a time, the beam's candidates of lines of the last run, broken().
// Built against the reference's headers by oracle/ref.mk (target `adapter`); run by
// tests/test_gpu_adapter.py, which compares what it writes with the reference's CPU path.
//
//   adapter_run <model blob> <input> <output>
//
// input (little-endian): int32 pages; per page int32 width, height, then its bytes; int32 groups;
// per group int32 count, its page indices, and per page int32 runs and [runs][2] int32 rows;
// int32 lines; per line int32 group, page (index into all pages), bucket width, float64 box[4];
// int32 rows, int32 topk, int32 rows[] (indices into the last recognize call's lines).
// output: per line int32 length, count, ids[count], frames[count], float32 probs[count]; int32 k;
// per row int32 frames, int32 ids[frames * k], float32 logp[frames * k], blank[frames]; int32
// broken; int32 1 when a recognize with another crop rule was refused.

#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <iterator>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "adapter.inc"

// The reference defines this in carbon/src/pipeline.cpp, which this driver does not link; the
// recognition path never calls it.
carbon::Tensor carbon::PipelineModels::detect_one(const Tensor&) { throw Error("detect_one: not on this path"); }

namespace {

struct Reader {
  std::vector<char> b;
  size_t at = 0;
  template <class T>
  T get() {
    T v;
    std::memcpy(&v, b.data() + at, sizeof(T));
    at += sizeof(T);
    return v;
  }
};

template <class T>
void put(std::ofstream& o, const T* p, size_t n) {
  o.write(reinterpret_cast<const char*>(p), static_cast<std::streamsize>(n * sizeof(T)));
}
template <class T>
void put1(std::ofstream& o, T v) {
  put(o, &v, 1);
}

}  // namespace

int main(int argc, char** argv) {
  if (argc != 4) {
    std::cerr << "usage: adapter_run <model blob> <input> <output>\n";
    return 2;
  }
  std::ifstream fb(argv[1], std::ios::binary), fi(argv[2], std::ios::binary);
  const std::string blob((std::istreambuf_iterator<char>(fb)), std::istreambuf_iterator<char>());
  Reader in{std::vector<char>((std::istreambuf_iterator<char>(fi)), std::istreambuf_iterator<char>())};
  const int npages = in.get<int32_t>();
  std::vector<std::vector<uint8_t>> bytes(npages);
  std::vector<carbon::GrayView> views(npages);
  for (int p = 0; p < npages; ++p) {
    const int w = in.get<int32_t>(), h = in.get<int32_t>();
    bytes[p].assign(in.b.begin() + in.at, in.b.begin() + in.at + static_cast<size_t>(w) * h);
    in.at += static_cast<size_t>(w) * h;
    views[p] = {bytes[p].data(), w, h, w};
  }
  const int ngroups = in.get<int32_t>();
  std::vector<std::vector<int>> group_pages(ngroups);
  std::vector<std::vector<carbon::RowRuns>> group_rows(ngroups);
  for (int g = 0; g < ngroups; ++g) {
    const int count = in.get<int32_t>();
    for (int i = 0; i < count; ++i) group_pages[g].push_back(in.get<int32_t>());
    for (int i = 0; i < count; ++i) {
      carbon::RowRuns r;
      const int runs = in.get<int32_t>();
      for (int k = 0; k < runs; ++k) {
        const int a = in.get<int32_t>(), b = in.get<int32_t>();
        r.emplace_back(a, b);
      }
      group_rows[g].push_back(r);
    }
  }
  const int nlines = in.get<int32_t>();
  std::vector<int> line_group(nlines), line_page(nlines), line_bw(nlines);
  std::vector<carbon::LineBox> line_box(nlines);
  for (int i = 0; i < nlines; ++i) {
    line_group[i] = in.get<int32_t>();
    line_page[i] = in.get<int32_t>();
    line_bw[i] = in.get<int32_t>();
    double b[4];
    for (double& v : b) v = in.get<double>();
    line_box[i] = {b[0], b[1], b[2], b[3]};
  }
  const int ncand = in.get<int32_t>(), topk = in.get<int32_t>();
  std::vector<int32_t> cand_rows(ncand);
  for (int& r : cand_rows) r = in.get<int32_t>();

  carbon::PipelineOptions opts;
  opts.gpu = 0;
  opts.line_batch = 512;
  opts.in_flight = 4;
  const carbon::CropRule crop;
  std::vector<carbon::CtcLine> results(nlines);
  std::vector<int32_t> result_len(nlines);
  std::vector<carbon::FrameCandidates> cands;
  int refused = 0, broken = 0;
  try {
    std::unique_ptr<carbon::PipelineModels> m = std::make_unique<carbon::B200RecModels>(nullptr, blob, opts, crop);
    auto group_views = [&](int g) {
      std::vector<carbon::GrayView> v;
      for (int p : group_pages[g]) v.push_back(views[p]);
      return v;
    };
    for (int g = 0; g < ngroups; ++g) {
      const std::vector<carbon::GrayView> gv = group_views(g);
      m->set_pages(gv, group_rows[g]);
      std::vector<carbon::GrayView> next;
      if (g + 1 < ngroups) {
        next = group_views(g + 1);
        m->prefetch_pages(next, group_rows[g + 1]);
      }
      std::map<int, std::vector<int>> buckets;  // bucket width -> the group's lines, in input order
      for (int i = 0; i < nlines; ++i)
        if (line_group[i] == g) buckets[line_bw[i]].push_back(i);
      for (const auto& [bw, idx] : buckets) {
        std::vector<int32_t> page_of;
        std::vector<carbon::LineBox> boxes;
        for (int i : idx) {
          int local = 0;
          while (group_pages[g][local] != line_page[i]) ++local;
          page_of.push_back(local);
          boxes.push_back(line_box[i]);
        }
        std::vector<carbon::CtcLine> lines;
        std::vector<int32_t> lengths;
        m->recognize(page_of, boxes, bw, crop, lines, lengths);
        for (size_t j = 0; j < idx.size(); ++j) {
          results[idx[j]] = lines[j];
          result_len[idx[j]] = lengths[j];
        }
      }
    }
    // the last recognize call's lines (the last group's widest bucket)
    if (!m->candidates(cand_rows, topk, cands)) {
      std::cerr << "candidates: none\n";
      return 1;
    }
    broken = m->broken() ? 1 : 0;
    carbon::CropRule other = crop;
    other.pad_v += 0.05;
    std::vector<carbon::CtcLine> lines;
    std::vector<int32_t> lengths;
    try {
      const std::vector<int32_t> page_of{0};
      const std::vector<carbon::LineBox> boxes{line_box[0]};
      m->recognize(page_of, boxes, line_bw[0], other, lines, lengths);
    } catch (const carbon::Error&) {
      refused = 1;
    }
  } catch (const std::exception& e) {
    std::cerr << "adapter_run: " << e.what() << "\n";
    return 1;
  }
  std::ofstream o(argv[3], std::ios::binary);
  for (int i = 0; i < nlines; ++i) {
    const carbon::CtcLine& l = results[i];
    put1<int32_t>(o, result_len[i]);
    put1<int32_t>(o, static_cast<int32_t>(l.ids.size()));
    put(o, l.ids.data(), l.ids.size());
    put(o, l.frames.data(), l.frames.size());
    put(o, l.probs.data(), l.probs.size());
  }
  put1<int32_t>(o, cands.empty() ? 0 : cands[0].k);
  for (const carbon::FrameCandidates& f : cands) {
    put1<int32_t>(o, f.frames);
    put(o, f.ids.data(), f.ids.size());
    put(o, f.logp.data(), f.logp.size());
    put(o, f.blank.data(), f.blank.size());
  }
  put1<int32_t>(o, broken);
  put1<int32_t>(o, refused);
  return o.good() ? 0 : 1;
}

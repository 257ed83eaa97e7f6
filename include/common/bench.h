// bench.h — throughput helpers and the CSV writer of the host harness. Same API as
// the reference's include/common/bench.h:10-47 (bandwidth_gbps, tflops, CsvWriter:
// header written only when the file is empty, rows appended and flushed).
#pragma once

#include <fstream>
#include <string>
#include <vector>

namespace hopper {

inline double bandwidth_gbps(double bytes, double ms) { return bytes / (ms * 1e6); }
inline double tflops(double flops, double ms) { return flops / (ms * 1e9); }

class CsvWriter {
 public:
  CsvWriter(std::string path, std::vector<std::string> columns)
      : path_(std::move(path)), columns_(std::move(columns)) {
    bool empty = true;
    {
      std::ifstream probe(path_);
      empty = !(probe.good() && probe.peek() != std::ifstream::traits_type::eof());
    }
    out_.open(path_, std::ios::app);
    if (empty) write(columns_);
  }
  void row(const std::vector<std::string>& values) { write(values); }

 private:
  void write(const std::vector<std::string>& v) {
    for (size_t i = 0; i < v.size(); ++i) out_ << (i ? "," : "") << v[i];
    out_ << '\n';
    out_.flush();
  }
  std::string path_;
  std::vector<std::string> columns_;
  std::ofstream out_;
};

}  // namespace hopper

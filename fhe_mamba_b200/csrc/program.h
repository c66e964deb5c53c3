// Packed-program executor: reads fhemamba's exported CKKS programs
// (`fhemamba-packed-v1` / `-v2`, grammar of the reference's
// native/fideslib_stage0/include/packed_program.hpp:60-163) and evaluates them
// node by node on the device, following PackedEvaluator::evaluate
// (native/fideslib_stage0/src/packed_fideslib.cpp:600-836) with the baseline
// refresh policy (refresh a parent whose level plus the node's need exceeds
// the refresh ceiling; one or two bootstrap passes).
#pragma once
#include <cstdint>
#include <functional>
#include <istream>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "bootstrap.h"
#include "ckks.h"

namespace fhe {

struct PackedNode {
  std::string op;
  int size = 0;
  double bound = 0;
  std::vector<int> parents;
  std::vector<double> data;
};

struct PackedOutput {
  int node = 0;
  std::vector<double> polynomial, exact;
};

struct PackedProgram {
  int version = 1;
  int slots = 0;
  double bound = 0;
  std::vector<PackedNode> nodes;
  std::vector<PackedOutput> outputs;
};

// Parses and validates a program; throws fhe::Error(-1) on malformed input.
PackedProgram read_packed_program(std::istream& in);

struct OutputErrors {
  double polynomial = 0, exact = 0;
  int non_finite = 0;
};
OutputErrors packed_output_errors(const std::vector<double>& values, const PackedOutput& ref);

// Client side of generation: the vocabulary head (u32 vocab, u32 width,
// f32[vocab * width], tied embedding) and the greedy selection.
struct GenerationClient {
  uint32_t vocab = 0, width = 0;
  std::vector<float> weights;
  std::vector<int> tokens;
  std::vector<double> margins;
  void load(const std::string& path);
  // argmax_token(hidden . W_token); returns that token's embedding row.
  std::vector<double> select(const std::vector<double>& hidden);
};

struct ExecutorOptions {
  int bootstrap_passes = 2;
  int refresh_margin = 5;       // refresh ceiling = max level - margin
  uint32_t max_rotation_keys = 512;  // beyond this, rotations decompose into powers of two
  bool trace = false;
};

struct OperationStats {
  long long nodes = 0, bootstraps = 0;
  double seconds = 0, bootstrap_seconds = 0;
};

class PackedExecutor {
 public:
  PackedExecutor(Ckks& ck, Bootstrapper* boot, const PackedProgram& program, const ExecutorOptions& opt);

  // Evaluates every node; returns the encrypted outputs in program order.
  std::vector<std::unique_ptr<Ct>> evaluate();
  std::vector<double> decrypt(const Ct& c, int count);

  std::function<std::unique_ptr<Ct>(const Ct&)> client_feedback;

  // counters (the reference's native.json fields)
  long long ct_ct = 0, ct_pt = 0, rotations = 0, adds = 0, bootstraps = 0, logical_refreshes = 0;
  long long rotation_keys_generated = 0;
  double bootstrap_seconds = 0, keygen_seconds = 0;
  int refresh_ceiling = 0, refreshed_level = -1;
  std::map<std::string, OperationStats> operation_stats;

  int level(const Ct& c) const { return (int)ck_.ctx.L - (int)c.nq; }
  std::unique_ptr<Ct> encrypt(const std::vector<double>& values);

 private:
  std::unique_ptr<Ct> plain(const Ct& a, std::vector<double> values, bool multiply);
  std::unique_ptr<Ct> rotate(const Ct& a, int offset);
  std::vector<std::unique_ptr<Ct>> rotate_many(const Ct& a, const std::vector<int>& offsets);
  std::unique_ptr<Ct> transform(const Ct& x, const std::map<int, std::vector<double>>& masks);
  std::unique_ptr<Ct> bsgs(const Ct& x, const std::map<int, std::vector<double>>& masks);
  std::unique_ptr<Ct> gather(const Ct& x, const std::vector<double>& indices, int size, bool scatter);
  std::unique_ptr<Ct> linear(const Ct& x, const PackedNode& weights, int columns);
  std::unique_ptr<Ct> chebyshev(const Ct& x, const PackedNode& node);
  std::unique_ptr<Ct> rotation_sum(const Ct& input, int count, int stride);
  std::unique_ptr<Ct> refresh(const Ct& value, double bound);
  std::unique_ptr<Ct> scale(const Ct& a, double c);
  std::unique_ptr<Ct> add(const Ct& a, const Ct& b, bool subtract = false);
  bool ensure_key(int step);

  Ckks& ck_;
  Bootstrapper* boot_;
  const PackedProgram& p_;
  ExecutorOptions opt_;
  uint32_t slots_;
};

}  // namespace fhe

// packed_b200: drop-in for the reference's packed_fideslib executable
// (native/fideslib_stage0/src/packed_fideslib.cpp:882-1403).  Same argv and
// exit codes: PROGRAM RESULT POLY_TOL EXACT_TOL [options]; 0 = passed,
// 1 = a gate failed, 2 = exception.  Options that only select among the
// reference's FIDESlib scheduling variants (hoisting, caches, plaintext upload
// paths, routing radix) are accepted and have no effect here; the ones that
// change the computation are honoured.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <iostream>
#include <set>
#include <string>

#include "fhe_b200.h"

int main(int argc, char** argv) {
  if (argc < 5) {
    std::cerr << "usage: packed_b200 PROGRAM RESULT POLY_TOL EXACT_TOL [--bootstrap-passes 1|2] "
                 "[--client-head FILE] [--trace-levels] [--s2c-first] [--ring-log N] [--depth D] [--seed S] "
                 "[--device D] [--secret-key-dist uniform-ternary|sparse-encapsulated] [--sparse-h H] "
                 "[--security not-set|128-classic] [--security-digits N]"
              << std::endl;
    return 2;
  }
  // scheduling variants of the reference executor: accepted, no effect
  static const std::set<std::string> no_effect = {
      "--direct-linear", "--legacy-routing", "--planned-refresh", "--batch-refresh",
      "--merge-refresh-correction", "--profile-evaluation", "--inplace-ops", "--naf-rotations",
      "--reuse-dead-inputs", "--reuse-public-ciphertexts", "--compact-weights", "--cache-plaintexts",
      "--indexed-mask-cache", "--prefetch-plaintexts", "--fast-plaintext-upload", "--direct-plaintext-upload",
      "--gpu-plaintext-ntt", "--move-plaintext-coefficients", "--borrow-plaintext-upload",
      "--bsgs-routing-stages", "--frontier-refresh", "--gpu-plaintext-rns", "--gpu-addend-rns",
      "--gpu-plaintext-fft", "--batch-plaintext-rns", "--fuse-plaintext-rns-ntt", "--hoist-rotations",
      "--share-chebyshev"};
  static const std::set<std::string> no_effect_with_value = {"--plaintext-cache-capacity", "--prefetch-workers",
                                                             "--frontier-live-limit"};
  fhe_program_options o{};
  std::string client;
  try {
    for (int i = 5; i < argc; ++i) {
      const std::string a = argv[i];
      auto value = [&]() -> std::string {
        if (i + 1 >= argc) throw std::invalid_argument("missing value for " + a);
        return argv[++i];
      };
      if (a == "--bootstrap-passes") {
        o.bootstrap_passes = std::stoi(value());
        if (o.bootstrap_passes != 1 && o.bootstrap_passes != 2)
          throw std::invalid_argument("bootstrap passes must be 1 or 2");
      } else if (a == "--client-head") {
        client = value();
      } else if (a == "--trace-levels") {
        o.trace = 1;
      } else if (a == "--s2c-first") {
        o.s2c_first = 1;
      } else if (a == "--ring-log") {
        o.log_n = (uint32_t)std::stoul(value());
      } else if (a == "--depth") {
        o.depth = (uint32_t)std::stoul(value());
      } else if (a == "--seed") {
        o.seed = std::stoull(value());
      } else if (a == "--device") {
        o.device = std::stoi(value());
      } else if (a == "--secret-key-dist") {
        // the decode driver's choices (stage1_mamba2_decode_fideslib.cpp:284-291);
        // bootstrapping under a sparse secret of weight 32 by encapsulation
        const std::string d = value();
        if (d == "sparse-encapsulated") o.sparse_h = o.sparse_h ? o.sparse_h : 32;
        else if (d == "uniform-ternary") o.sparse_h = 0;
        else throw std::invalid_argument("secret key distribution must be uniform-ternary or sparse-encapsulated");
      } else if (a == "--sparse-h") {
        o.sparse_h = (uint32_t)std::stoul(value());
      } else if (a == "--security") {
        const std::string v = value();
        if (v == "128-classic") o.security128 = 1;
        else if (v != "not-set") throw std::invalid_argument("security must be not-set or 128-classic");
      } else if (a == "--security-digits") {
        o.security_digits = (uint32_t)std::stoul(value());
      } else if (no_effect.count(a)) {
      } else if (no_effect_with_value.count(a)) {
        value();
      } else {
        throw std::invalid_argument("unknown packed option: " + a);
      }
    }
    const double poly_tol = std::stod(argv[3]), exact_tol = std::stod(argv[4]);
    const int rc = fhe_program_run(argv[1], client.empty() ? nullptr : client.c_str(), argv[2], poly_tol,
                                   exact_tol, &o);
    if (rc < 0) {
      char msg[1024];
      fhe_last_error(msg, sizeof msg);
      std::cerr << msg << std::endl;
      return 2;
    }
    return rc;
  } catch (const std::exception& e) {
    std::cerr << e.what() << std::endl;
    return 2;
  }
}

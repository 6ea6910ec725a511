// Driver program over the reference's own launch contract (compiled from
// its source by oracle/Makefile into oracle/_ref/).  Test infrastructure
// only: the tests feed it cases on stdin and compare its verdicts and
// messages with ours.  It runs as its own process.
//
// Input, one case per line:
//   G gx gy gz bx by bz smem uses_cluster cx cy cz
//   L storage_size misalign null_storage n_offsets n_codes off... code...
// Output per case: "OK" or "ERR <message>".
#include <cstdint>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "flight4s/cuda/launch_contract.hpp"

int main() {
  alignas(16) static unsigned char storage[512];
  std::string line;
  while (std::getline(std::cin, line)) {
    std::istringstream in(line);
    char kind = 0;
    in >> kind;
    std::optional<std::string> error;
    if (kind == 'G') {
      int v[11];
      for (int& x : v) in >> x;
      const flight4s::cuda::LaunchGeometry g{v[0], v[1], v[2], v[3], v[4], v[5], v[6], v[7] != 0, v[8], v[9], v[10]};
      error = flight4s::cuda::validate_launch_geometry(g);
    } else if (kind == 'L') {
      long long size = 0;
      int misalign = 0, null_storage = 0;
      std::size_t n_off = 0, n_code = 0;
      in >> size >> misalign >> null_storage >> n_off >> n_code;
      std::vector<std::int32_t> offsets(n_off);
      std::vector<std::int8_t> codes(n_code);
      for (auto& o : offsets) in >> o;
      for (auto& c : codes) {
        int x;
        in >> x;
        c = static_cast<std::int8_t>(x);
      }
      const flight4s::cuda::ArgumentLayout l{null_storage ? nullptr : storage + misalign, size,
                                             offsets.empty() ? nullptr : offsets.data(), n_off,
                                             codes.empty() ? nullptr : codes.data(), n_code};
      error = flight4s::cuda::validate_argument_layout(l);
    } else {
      continue;
    }
    if (error) std::cout << "ERR " << *error << "\n"; else std::cout << "OK\n";
  }
  return 0;
}

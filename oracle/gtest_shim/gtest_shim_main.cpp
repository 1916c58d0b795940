// main() for the GoogleTest-compatible shim: runs every registered TEST,
// prints one line per test and a summary line
//   SUMMARY passed=P failed=F skipped=S
// and returns non-zero if any test failed.  Test infrastructure only.
#include <gtest/gtest.h>

#include <cstring>
#include <exception>

int main(int argc, char** argv) {
  const char* filter = argc > 1 ? argv[1] : nullptr;
  int passed = 0, failed = 0, skipped = 0;
  for (const auto& t : gtest_shim::registry()) {
    const std::string full = std::string(t.suite) + "." + t.name;
    if (filter && full.find(filter) == std::string::npos) continue;
    auto& s = gtest_shim::state();
    s.failed = false;
    s.skipped = false;
    try {
      t.fn();
    } catch (const std::exception& e) {
      std::cerr << full << ": uncaught exception: " << e.what() << "\n";
      s.failed = true;
    } catch (...) {
      std::cerr << full << ": uncaught exception\n";
      s.failed = true;
    }
    const char* verdict = s.failed ? "FAILED" : (s.skipped ? "SKIPPED" : "OK");
    std::cout << "[" << verdict << "] " << full << std::endl;
    if (s.failed) ++failed;
    else if (s.skipped) ++skipped;
    else ++passed;
  }
  std::cout << "SUMMARY passed=" << passed << " failed=" << failed
            << " skipped=" << skipped << std::endl;
  return failed ? 1 : 0;
}

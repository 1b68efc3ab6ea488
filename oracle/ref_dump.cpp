// ORACLE — test infrastructure.  Prints the graphs PyFlame's own front end
// builds (ref_build in ref_shim.cpp) for each kind given on the command line,
// separated by lines of "----".  Runs as its own process so no other library
// shares its address space.
#include <cstdio>
#include <cstdlib>

extern "C" int ref_build(int kind, char* buf, unsigned long len);
extern "C" const char* ref_last_error(void);

int main(int argc, char** argv) {
  static char buf[1 << 20];
  for (int i = 1; i < argc; ++i) {
    if (ref_build(std::atoi(argv[i]), buf, sizeof buf) != 0) {
      std::fprintf(stderr, "%s\n", ref_last_error());
      return 1;
    }
    std::printf("%s----\n", buf);
  }
  return 0;
}

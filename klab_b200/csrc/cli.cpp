// bin/klab: native launcher of the command-line runner (drop-in for the reference's
// native/cli.cpp, which execs experiments.py). It finds the project, picks the Python
// interpreter and replaces itself with `python -m klab_b200.cli <args>`, so the runner's
// exit status is the launcher's.
//
// Project root, first match: `--project <dir>` before the command; $KERNEL_LAB_ROOT; the
// directory above this executable's own directory (bin/..); the root baked in at build time.
// A directory is a project when it holds klab_b200/cli.py and klab_b200/kernel_lab.py.
// Interpreter, first match: <root>/.venv/bin/python; $KLAB_PYTHON; the one baked in at build
// time (the interpreter that ran the build); python3 on PATH.
// Errors of the launcher itself print "klab: ..." and exit 2.
#include <cerrno>
#include <climits>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <iostream>
#include <stdexcept>
#include <string>
#include <unistd.h>
#include <vector>

namespace fs = std::filesystem;

#ifndef KLAB_PROJECT_ROOT
#define KLAB_PROJECT_ROOT ""
#endif
#ifndef KLAB_PYTHON
#define KLAB_PYTHON ""
#endif

namespace {

bool is_project(const fs::path& dir) {
  std::error_code ec;
  return fs::is_regular_file(dir / "klab_b200" / "cli.py", ec) && fs::is_regular_file(dir / "klab_b200" / "kernel_lab.py", ec);
}

fs::path self_root() {
  char buf[PATH_MAX];
  const ssize_t n = readlink("/proc/self/exe", buf, sizeof(buf) - 1);
  if (n <= 0) return {};
  buf[n] = '\0';
  return fs::path(buf).parent_path().parent_path();
}

bool executable(const fs::path& p) {
  std::error_code ec;
  return fs::is_regular_file(p, ec) && access(p.c_str(), X_OK) == 0;
}

}  // namespace

int main(int argc, char** argv) {
  try {
    int first = 1;
    fs::path root;
    bool explicit_root = false;
    if (argc > 1 && std::string(argv[1]) == "--project") {
      if (argc < 3) throw std::runtime_error("usage: klab --project <directory> <command>");
      root = argv[2];
      first = 3;
      explicit_root = true;
    } else if (const char* env = std::getenv("KERNEL_LAB_ROOT")) {
      root = env;
      explicit_root = true;
    } else {
      root = self_root();
      if (root.empty() || !is_project(root)) root = KLAB_PROJECT_ROOT;
    }
    std::error_code ec;
    root = fs::canonical(root, ec);
    if (ec || !is_project(root))
      throw std::runtime_error((root.empty() ? std::string("<none>") : root.string()) + " is not a klab-b200 project" +
                               (explicit_root ? "" : " (pass --project <directory>)"));
    std::string python;
    if (executable(root / ".venv" / "bin" / "python")) {
      python = (root / ".venv" / "bin" / "python").string();
    } else if (const char* env = std::getenv("KLAB_PYTHON")) {
      python = env;
    } else if (executable(KLAB_PYTHON)) {
      python = KLAB_PYTHON;
    } else {
      python = "python3";
    }
    std::vector<std::string> words{python, "-m", "klab_b200.cli"};
    for (int i = first; i < argc; ++i) words.emplace_back(argv[i]);
    std::vector<char*> args;
    for (auto& w : words) args.push_back(w.data());
    args.push_back(nullptr);
    fs::current_path(root);
    if (python.find('/') == std::string::npos)
      execvp(python.c_str(), args.data());
    else
      execv(python.c_str(), args.data());
    throw std::runtime_error("cannot start " + python + ": " + std::strerror(errno));
  } catch (const std::exception& error) {
    std::cerr << "klab: " << error.what() << '\n';
    return 2;
  }
}

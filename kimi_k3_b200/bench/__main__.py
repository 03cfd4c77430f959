"""``python -m kimi_k3_b200.bench <name> [options]``."""
import sys


def main(argv=None):
    argv = list(sys.argv[1:] if argv is None else argv)
    if not argv or argv[0] in ("-h", "--help"):
        from . import modules
        print("usage: python -m kimi_k3_b200.bench {kernels <case>|" + "|".join(sorted(modules.BENCHMARKS)) + "} ...")
        return 0
    name, rest = argv[0], argv[1:]
    if name == "kernels":
        from . import kernels
        kernels.main(rest)
        return 0
    from . import modules
    if name not in modules.BENCHMARKS:
        raise SystemExit(f"unknown benchmark {name!r}")
    modules.BENCHMARKS[name](rest)
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""``python -m sigma0_b200.cli {train,infer,plan,launch,rl} ...``"""
import sys

_COMMANDS = ("train", "infer", "plan", "launch", "rl")


def main():
    if len(sys.argv) < 2 or sys.argv[1] not in _COMMANDS:
        print("usage: python -m sigma0_b200.cli {train,infer,plan,launch,rl} [args]", file=sys.stderr)
        return 2
    cmd, rest = sys.argv[1], sys.argv[2:]
    if cmd == "train":
        from .train import main as m
    elif cmd == "infer":
        from .infer import main as m
    elif cmd == "launch":
        from .launch import main as m
    elif cmd == "rl":
        from .rl import main as m
    else:
        from .plan import main as m
    return m(rest)


if __name__ == "__main__":
    raise SystemExit(main())

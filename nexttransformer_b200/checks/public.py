"""Scan tracked files for content that does not belong in a public repository.

    python -m nexttransformer_b200.checks.public            # every tracked file
    python -m nexttransformer_b200.checks.public PATH ...   # only these files

Flags credentials and tokens, private keys, absolute paths into personal home directories, personal
e-mail addresses and private-network IP addresses.  Exits non-zero on a finding.  The loopback
rendezvous address used by the launch helpers is not a private-network address.
Behaviour: ``nexttransformer/checks/public.py`` of the reference (same categories).
"""
import re
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[2]
TOKEN = re.compile(r"\b(?:gh[pousr]_[A-Za-z0-9]{36,}|github_pat_[A-Za-z0-9_]{50,}|hf_[A-Za-z0-9]{34,}|sk-[A-Za-z0-9]{32,}"
                   r"|AKIA[0-9A-Z]{16}|xox[abprs]-[A-Za-z0-9-]{10,})\b|-----BEGIN [A-Z ]*PRIVATE KEY-----")
HOME = re.compile(r"/home/(?!runner/)[a-z_][a-z0-9_.-]*/|/Users/[A-Za-z][^/\s]*/|[A-Z]:\\Users\\")
MAIL = re.compile(r"\b[A-Za-z0-9._%+-]{2,}@[A-Za-z0-9-]{2,}(?:\.[A-Za-z0-9-]+)*\.[A-Za-z]{2,6}\b")
MAIL_OK = re.compile(r"(?:noreply|no-reply)@|@users\.noreply\.github\.com|@example\.(?:com|org|net)$")
LAN = re.compile(r"\b(?:10\.\d{1,3}\.\d{1,3}\.\d{1,3}|192\.168\.\d{1,3}\.\d{1,3}|172\.(?:1[6-9]|2\d|3[01])\.\d{1,3}\.\d{1,3})\b")
SKIP_SUFFIX = (".png", ".jpg", ".jpeg", ".pdf", ".pt", ".so", ".lock")
SELF = "nexttransformer_b200/checks/public.py"


def tracked():
    out = subprocess.run(["git", "ls-files"], cwd=REPO, capture_output=True, text=True, check=True).stdout
    return out.splitlines()


def scan_text(path, text):
    found = []
    for n, line in enumerate(text.splitlines(), 1):
        hits = ["possible credential (redacted)"] if TOKEN.search(line) else []
        hits += [m.group(0) for m in HOME.finditer(line)]
        hits += [m.group(0) for m in MAIL.finditer(line) if not MAIL_OK.search(m.group(0))]
        hits += [m.group(0) for m in LAN.finditer(line)]
        found += [f"{path}:{n}: {h}" for h in hits]
    return found


def scan(paths):
    found = []
    for path in paths:
        f = REPO / path
        if path == SELF or path.endswith(SKIP_SUFFIX) or not f.is_file():
            continue
        try:
            found += scan_text(path, f.read_text())
        except UnicodeDecodeError:
            continue
    return found


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    found = scan(argv or tracked())
    print("\n".join(found) if found else "no findings")
    raise SystemExit(1 if found else 0)


if __name__ == "__main__":
    main()

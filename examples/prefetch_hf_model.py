#!/usr/bin/env python
"""Download a Hugging Face model snapshot ahead of a run (safetensors + config).

Counterpart of the reference's ``prefetch_hf_model.py``.  The files land in the
Hugging Face cache (or ``--local-dir``) so the trainers can stream them with
``--checkpoint``.  Needs network access to the Hub.

    python examples/prefetch_hf_model.py --model Qwen/Qwen2.5-7B --local-dir /data/qwen7b
"""

from __future__ import annotations

import argparse
import sys


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    p.add_argument("--model", required=True, help="Hub repo id, e.g. Qwen/Qwen2.5-1.5B")
    p.add_argument("--revision", default=None)
    p.add_argument("--local-dir", default=None)
    p.add_argument("--allow", nargs="*", default=["*.safetensors", "*.json", "tokenizer*"],
                   help="file patterns to fetch")
    args = p.parse_args(argv)
    try:
        from huggingface_hub import snapshot_download
    except ImportError:
        print("huggingface_hub is not installed", file=sys.stderr)
        return 2
    try:
        path = snapshot_download(repo_id=args.model, revision=args.revision,
                                 local_dir=args.local_dir, allow_patterns=args.allow)
    except Exception as e:  # no network, unknown repo, auth
        print(f"download failed: {type(e).__name__}: {e}", file=sys.stderr)
        return 1
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())

"""Download pre-tokenised GPT-2 shards of the fineweb10B corpus from the HuggingFace hub instead of re-tokenising
(`data/cached_fineweb10B.py` and siblings in the reference):  python data/cached_fineweb10B.py [num_train_shards]
Each shard holds 100M tokens; shard 0 is the validation split.  Needs network access and `huggingface_hub`."""
import os
import sys


def fetch(name: str, local_dir: str):
    if os.path.exists(os.path.join(local_dir, name)):
        return
    from huggingface_hub import hf_hub_download
    hf_hub_download(repo_id="kjj0/fineweb10B-gpt2", filename=name, repo_type="dataset", local_dir=local_dir)


def main():
    local_dir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "fineweb10B")
    count = int(sys.argv[1]) if len(sys.argv) > 1 else 103
    fetch("fineweb_val_%06d.bin" % 0, local_dir)
    for i in range(1, count + 1):
        fetch("fineweb_train_%06d.bin" % i, local_dir)


if __name__ == "__main__":
    main()

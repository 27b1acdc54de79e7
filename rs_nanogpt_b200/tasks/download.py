"""SFT dataset manifest (rs-nanogpt src/tasks/download.rs:21-85)."""
from ..data.download import FileJob, Summary, download_files

HF = "https://huggingface.co/datasets"
IDENTITY_URL = "https://karpathy-public.s3.us-west-2.amazonaws.com/identity_conversations.jsonl"
SFT_FILES = [
    ("HuggingFaceTB/smol-smoltalk/resolve/main/data/train-00000-of-00004.parquet", "smoltalk-train-00000.parquet"),
    ("HuggingFaceTB/smol-smoltalk/resolve/main/data/train-00001-of-00004.parquet", "smoltalk-train-00001.parquet"),
    ("HuggingFaceTB/smol-smoltalk/resolve/main/data/train-00002-of-00004.parquet", "smoltalk-train-00002.parquet"),
    ("HuggingFaceTB/smol-smoltalk/resolve/main/data/train-00003-of-00004.parquet", "smoltalk-train-00003.parquet"),
    ("HuggingFaceTB/smol-smoltalk/resolve/main/data/test-00000-of-00001.parquet", "smoltalk-test-00000.parquet"),
    ("cais/mmlu/resolve/main/all/auxiliary_train-00000-of-00001.parquet", "mmlu-train-00000.parquet"),
    ("cais/mmlu/resolve/main/all/test-00000-of-00001.parquet", "mmlu-test-00000.parquet"),
    ("openai/gsm8k/resolve/main/main/train-00000-of-00001.parquet", "gsm8k-train-00000.parquet"),
    ("openai/gsm8k/resolve/main/main/test-00000-of-00001.parquet", "gsm8k-test-00000.parquet"),
]


def sft_jobs():
    jobs = [FileJob(f"{HF}/{p}", f) for p, f in SFT_FILES]
    jobs.append(FileJob(IDENTITY_URL, "identity_conversations.jsonl"))
    return jobs


def download_sft_data(directory: str, workers: int) -> Summary:
    return download_files(directory, sft_jobs(), workers)

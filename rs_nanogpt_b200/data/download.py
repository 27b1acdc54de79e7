"""Dataset downloads (rs-nanogpt src/data/download.rs:11-218): parallel
workers, files already on disk are skipped, each download streams to
``<name>.tmp`` and is renamed into place atomically, 5 attempts with
1 s * 2^attempt back-off, 30 s connect/read timeouts."""
import os
import time
import urllib.request
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import List, Optional

MAX_SHARD = 6542
ATTEMPTS = 5


@dataclass
class FileJob:
    url: str
    filename: str


@dataclass
class Summary:
    requested: int = 0
    downloaded: int = 0
    skipped: int = 0
    failed: int = 0


def shard_name(i: int) -> str:
    return f"shard_{i:05d}.parquet"


def _fetch(job: FileJob, directory: str, backoff_s: float) -> str:
    dest = os.path.join(directory, job.filename)
    if os.path.exists(dest):
        return "skipped"
    tmp = dest + ".tmp"
    for attempt in range(ATTEMPTS):
        try:
            with urllib.request.urlopen(job.url, timeout=30) as r, open(tmp, "wb") as f:
                while True:
                    chunk = r.read(1 << 20)
                    if not chunk:
                        break
                    f.write(chunk)
            os.replace(tmp, dest)
            return "downloaded"
        except Exception as e:  # network errors, HTTP errors
            if os.path.exists(tmp):
                os.remove(tmp)
            if attempt + 1 == ATTEMPTS:
                print(f"failed {job.url}: {e}")
                return "failed"
            time.sleep(backoff_s * (2 ** attempt))
    return "failed"


def download_files(directory: str, jobs: List[FileJob], workers: int, backoff_s: float = 1.0) -> Summary:
    os.makedirs(directory, exist_ok=True)
    s = Summary(requested=len(jobs))
    with ThreadPoolExecutor(max_workers=workers) as pool:
        for res in pool.map(lambda j: _fetch(j, directory, backoff_s), jobs):
            setattr(s, res, getattr(s, res) + 1)
    return s


def download_shards(directory: str, start: int, num: int, val_shard: Optional[int], workers: int,
                    base_url: str, backoff_s: float = 1.0) -> Summary:
    idx = list(range(start, start + num))
    if val_shard is not None and val_shard not in idx:
        idx.append(val_shard)
    jobs = [FileJob(f"{base_url.rstrip('/')}/{shard_name(i)}", shard_name(i)) for i in idx]
    return download_files(directory, jobs, workers, backoff_s)

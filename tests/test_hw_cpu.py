"""GPU detection and KV calibration logic on the host (a fake device list, an injected survival
test): the reference's gpu-detect.sh TP rule and calibrate-kv.sh search."""
from vllm_sly_radiance_b200.config import get_model_config
from vllm_sly_radiance_b200.entrypoints.hw import (GpuInfo, detect_gpus, lookup_pin, pick_tp,
                                                  save_pin, search_blocks)


def test_tp_pick_follows_head_divisibility():
    m = get_model_config("qwen38_27b")       # 24 q / 4 kv heads, GDN 16 k / 48 v
    assert pick_tp(8, m) == 8
    assert pick_tp(7, m) == 4 and pick_tp(3, m) == 2 and pick_tp(1, m) == 1
    assert pick_tp(8, m, allowed=(6, 1)) == 1          # 6 does not divide the GDN key heads


def test_detect_skips_small_devices(tmp_path):
    m = get_model_config("qwen38_27b")
    gpus = [GpuInfo(0, "NVIDIA B200", 183359), GpuInfo(1, "tiny display", 2048),
            GpuInfo(2, "NVIDIA B200", 183359)]
    d = detect_gpus(m, gpus)
    assert [g["index"] for g in d["gpus"]] == [0, 2] and d["tensor_parallel_size"] == 2
    assert [g["index"] for g in d["skipped"]] == [1]


def test_kv_search_and_profile_table(tmp_path):
    limit = 7777
    tries = []

    def survives(n):
        tries.append(n)
        return n <= limit
    got = search_blocks(survives, 1024, tol=16)
    assert limit - 16 <= got <= limit and len(tries) < 30
    assert search_blocks(lambda n: n <= 300, 1024, tol=8) >= 292
    p = str(tmp_path / "kv.tsv")
    save_pin("NVIDIA B200", "qwen38_27b", 1, 8, 4096, got, p)
    save_pin("NVIDIA B200", "qwen38_27b", 2, 8, 4096, 9999, p)
    save_pin("NVIDIA B200", "qwen38_27b", 1, 8, 4096, got - 1, p)     # replaces the row
    assert lookup_pin("NVIDIA B200", "qwen38_27b", 1, 8, 4096, p) == got - 1
    assert lookup_pin("NVIDIA B200", "qwen38_27b", 2, path=p) == 9999
    assert lookup_pin("NVIDIA H100", "qwen38_27b", 1, path=p) is None

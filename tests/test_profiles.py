"""CPU: the measurement data bench.py reads from profiles/.

bench.py fills its `roofline.traffic` field (DRAM bytes per launch of the
dominant kernel) from profiles/roofline_traffic.json, keyed
"<workload>/<kernel>"; each entry names the ncu summary it was taken from.
These checks keep that file and the summaries it cites consistent.
"""
import json
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
TRAFFIC = ROOT / "profiles" / "roofline_traffic.json"


def test_traffic_entries_are_positive_and_cite_a_summary():
    data = json.loads(TRAFFIC.read_text())
    entries = {k: v for k, v in data.items() if not k.startswith("_")}
    # the config-2 kernels, one of which is the dominant kernel of the default bench line
    for kernel in ("attn_bwd_dkdv_sm100", "attn_fwd_sm100", "attn_bwd_dq_sm100"):
        assert f"config2/{kernel}" in entries
    for key, entry in entries.items():
        assert entry["dram_bytes_per_launch"] > 0, key
        source = ROOT / entry["source"]
        assert source.is_file(), (key, entry["source"])
        assert source.suffix in (".md", ".txt"), key


def test_profile_summaries_are_text_and_give_their_command():
    for path in sorted((ROOT / "profiles").iterdir()):
        if path.name == TRAFFIC.name:
            continue
        assert path.suffix in (".md", ".txt"), path.name
        text = path.read_text()
        assert "Command" in text and "bench.py" in text, path.name
        # every ncu command leaves the GPU clocks alone
        for line in text.splitlines():
            if line.lstrip().startswith("ncu --"):
                assert "--clock-control none" in line, (path.name, line)

"""ncu_sweep's CSV parsing (the GPU sweep itself runs only on a B200)."""
import math

from attnprofile_b200 import ncu_sweep

SAMPLE = '''==PROF== Connected to process 123
"ID","Process ID","Process Name","Host Name","Kernel Name","Context","Stream","Block Size","Grid Size","Device","CC","Section Name","Metric Name","Metric Unit","Metric Value"
"0","123","python","127.0.0.1","attn_fwd_kernel","1","7","(384, 1, 1)","(256, 1, 1)","0","10.0","Command line profiler metrics","dram__bytes_read.sum","Mbyte","50.39"
"0","123","python","127.0.0.1","attn_fwd_kernel","1","7","(384, 1, 1)","(256, 1, 1)","0","10.0","Command line profiler metrics","gpu__time_duration.sum","usecond","143.30"
"0","123","python","127.0.0.1","attn_fwd_kernel","1","7","(384, 1, 1)","(256, 1, 1)","0","10.0","Command line profiler metrics","sm__pipe_tensor_cycles_active.avg.pct_of_peak_sustained_active","%","59.38"
'''


def test_parse_ncu_csv_units():
    m = ncu_sweep.parse_ncu_csv(SAMPLE)
    assert math.isclose(m["time"], 0.1433)            # ms
    assert math.isclose(m["dram_read_bytes"], 50.39e6)
    assert math.isclose(m["tc_utilization"], 59.38)
    assert "xu_utilization" not in m


def test_parse_ncu_csv_empty():
    assert ncu_sweep.parse_ncu_csv("no csv here") == {}


def test_parse_shapes():
    assert ncu_sweep.parse_shapes("1x32x8192x128:bf16, 1x8x32768x128") == [
        (1, 32, 8192, 128, "bf16"), (1, 8, 32768, 128, "f16")]

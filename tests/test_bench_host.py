"""Host-side helpers of bench.py (no GPU): the ncu-CSV traffic reader and the
input generators' shapes."""

import bench


def test_ncu_traffic_per_attention_call(tmp_path):
    hdr = '"ID","Kernel Name","Metric Name","Metric Unit","Metric Value"\n'
    rows = []
    for call in range(2):
        for k, rd, wr in (("attn::dq_scores_kernel<128>", 500e6, 8e6), ("attn::dq_pv_kernel<128>", 560e6, 4e6),
                          ("gemm::gemm_kc_kernel<64>", 35e6, 0)):
            rows.append(f'"{call}","{k}","dram__bytes_read.sum","byte","{rd:.0f}"\n')
            rows.append(f'"{call}","{k}","dram__bytes_write.sum","byte","{wr:.0f}"\n')
    p = tmp_path / "l.csv"
    p.write_text("==PROF== header line\n" + hdr + "".join(rows))
    assert bench._ncu_traffic(str(p)) == int(500e6 + 8e6 + 560e6 + 4e6)
    assert bench._ncu_traffic(None) is None


def test_attention_inputs_shape_and_pool_permutation():
    d = bench.attention_inputs(seed=2, batch=4, heads=8, kv_heads=2, head_dim=64, pool=200,
                               ctx_lo=16, ctx_hi=300)
    assert d["Q"].shape == (4, 8, 64) and d["KV"].shape == (200, 2, 16, 2, 64)
    used = []
    for r in range(4):
        n = (int(d["seq_lens"][r]) + 15) // 16
        used += d["bt"][r, :n].tolist()
    assert len(set(used)) == len(used) and all(0 <= b < 200 for b in used)

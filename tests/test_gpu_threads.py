"""Concurrent host threads on one device.

whisper.rs calls attention from several WhisperStates at once that share one
context (crates/ffi/src/lib.rs:1435-1455), so the library must be re-entrant:
its per-thread workspaces and error state, the mutex-guarded one-time set-up
(status word, tensor-map encoder, cluster occupancy) and its kernels on
separate streams. Four threads, each with its own stream, run bf16 and f32
encoder attention and f16 decode calls on their own inputs, several times
over, and every result is checked against the oracle computed beforehand.
"""
import threading

import pytest

from tests.helpers import check_16bit, check_f32, randn

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def W():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    import wattn
    return wattn


def test_four_threads_own_streams(W, oracle):
    import torch
    n_threads, reps = 4, 6
    bt, tt, ht = 2, 300, 4        # bf16 encoder calls
    tf, hf = 600, 2               # f32 calls (key splits in clusters of 2)
    ng, gs, tk, hd = 3, 5, 700, 4  # f16 decode calls
    cases = []
    for i in range(n_threads):
        d = ht * 64
        qb, kb, vb = (randn(1000 + 10 * i + s, bt * tt * d) for s in range(3))
        qb, kb, vb = (torch.from_numpy(x).to(torch.bfloat16) for x in (qb, kb, vb))
        ref_b = oracle.flash_attention_2_batched(qb.float().numpy(), kb.float().numpy(),
                                                 vb.float().numpy(), bt, tt, tt, ht, d, False)
        df = hf * 64
        qf, kf, vf = (randn(2000 + 10 * i + s, tf * df) for s in range(3))
        ref_f = oracle.flash_attention_2(qf, kf, vf, tf, tf, hf, df, False)
        dd = hd * 64
        qd = torch.from_numpy(randn(3000 + 10 * i, ng * gs * dd)).half()
        kd, vd = (torch.from_numpy(randn(3001 + 10 * i + s, ng * tk * dd)).half() for s in range(2))
        ref_d = oracle.decode_grouped(qd.float().numpy(), kd.float().numpy(), vd.float().numpy(),
                                      ng, gs, tk, hd, dd)
        cases.append(dict(
            b=tuple(x.cuda() for x in (qb, kb, vb)), ref_b=ref_b,
            f=tuple(torch.from_numpy(x).cuda() for x in (qf, kf, vf)), ref_f=ref_f,
            d=tuple(x.cuda() for x in (qd, kd, vd)), ref_d=ref_d))
    torch.cuda.synchronize()
    errors = []
    results = [None] * n_threads

    def work(i):
        try:
            torch.cuda.set_device(0)
            st = torch.cuda.Stream()
            c = cases[i]
            ob = torch.empty(bt * tt * ht * 64, dtype=torch.float32, device="cuda")
            of = torch.empty(tf * hf * 64, dtype=torch.float32, device="cuda")
            od = torch.empty(ng * gs * hd * 64, dtype=torch.float32, device="cuda")
            outs = []
            for _ in range(reps):
                with torch.cuda.stream(st):
                    W.attention_fwd(*c["b"], ob, batch=bt, t_q=tt, t_kv=tt, n_heads=ht,
                                    scale=0.125, stream=st)
                    W.attention_fwd(*c["f"], of, batch=1, t_q=tf, t_kv=tf, n_heads=hf,
                                    scale=0.125, stream=st)
                    W.decode_fwd(*c["d"], od, n_groups=ng, group_size=gs, t_kv=tk, n_heads=hd,
                                 scale=0.125, stream=st)
                st.synchronize()
                outs.append((ob.cpu().numpy(), of.cpu().numpy(), od.cpu().numpy()))
            results[i] = outs
        except Exception as e:  # reported on the main thread
            errors.append(repr(e))

    threads = [threading.Thread(target=work, args=(i,)) for i in range(n_threads)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=120)
    assert not errors, errors
    assert all(not t.is_alive() for t in threads)
    for i, outs in enumerate(results):
        assert outs is not None and len(outs) == reps
        for r, (ob, of, od) in enumerate(outs):
            check_16bit(ob, cases[i]["ref_b"], f"thread {i} rep {r} bf16")
            check_f32(of, cases[i]["ref_f"], f"thread {i} rep {r} f32")
            check_16bit(od, cases[i]["ref_d"], f"thread {i} rep {r} decode")
    assert W.device_status() == 0

"""Multi-GPU parity of the head-sharded prefill and batched decode.

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \
        --master-addr 127.0.0.1 --master-port P tests/mgpu_parity.py

Every rank builds the same seeded full inputs, runs its KV-head group
through the C ABI, and the outputs are all-gathered and head-concatenated
on every rank over NCCL (eyebrowse_b200.sharded.gather_heads). Rank 0 checks
the full result against the oracle at max-abs <= 2e-3, rel-L2 <= 1e-3. The
prefill then runs again with the gather fused into the attention kernel
(eb_attention_prefill_gather: TMA stores into every rank's symmetric-memory
buffer), and with own-buffer writes followed by eb_head_broadcast through
the NVLink multicast address; every rank checks that its gathered copy
equals the NCCL result bit for bit. The batched decode runs the same way,
then with the gather fused into the decode kernel
(eb_attention_decode_batched_gather): split by KV-head group it must equal
the NCCL result bit for bit, split by sequence (eyebrowse_b200.sharded.
decode_shard with one head group) it is checked against the oracle. Exits
non-zero on any mismatch. tests/test_gpu_multi.py runs it on 2 GPUs when a
machine has them.
"""
import datetime
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> int:
    import torch
    import torch.distributed as dist

    import eyebrowse_b200 as eb
    from eyebrowse_b200.sharded import (GatheredOutput, decode_shard, gather_heads,
                                        head_shard)
    from oracle import oracle as orc
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", local))
    ok = True
    # ---- prefill: config-3 geometry at S=4608 (f16): with 16 heads per rank
    # the grid is large enough for the two-tile (GQA pair) kernel
    S, H, Hkv, hd = 4608, 32, 8, 128
    rng = np.random.default_rng(11)
    q = orc.round_f16(rng.standard_normal((S, H, hd)).astype(np.float32) * 0.5).reshape(S, H, hd)
    k = orc.round_f16(rng.standard_normal((S, Hkv, hd)).astype(np.float32) * 0.5).reshape(S, Hkv, hd)
    v = orc.round_f16(rng.standard_normal((S, Hkv, hd)).astype(np.float32) * 0.5).reshape(S, Hkv, hd)
    cos, sin = eb.rope_tables(S, hd, 5e5)
    sh = head_shard(H, Hkv, world, rank)
    f16 = torch.float16
    dev = lambda x: torch.from_numpy(np.ascontiguousarray(x)).to(f16).cuda()
    desc = eb.make_desc(sh.n_heads, sh.n_kv_heads, hd, S, dtype_qkv=eb.EB_F16,
                        dtype_cache=eb.EB_F16, dtype_out=eb.EB_F16)
    layer = eb.make_layer(rope_cos=torch.from_numpy(cos).cuda(), rope_sin=torch.from_numpy(sin).cuda())
    kc = torch.empty(S, sh.n_kv_heads, hd, device="cuda", dtype=f16)
    vc = torch.empty_like(kc)
    o = torch.empty(S, sh.n_heads, hd, device="cuda", dtype=f16)
    ws = eb.alloc_workspace(eb.attention_prefill_workspace_bytes(desc, S))
    eb.attention_prefill(desc, layer, S, dev(q[:, sh.h0:sh.h1]), dev(k[:, sh.kv0:sh.kv1]),
                         dev(v[:, sh.kv0:sh.kv1]), kc, vc, o, ws)
    gath = torch.empty(world, S, sh.n_heads, hd, device="cuda", dtype=f16)
    full = torch.empty(S, H, hd, device="cuda", dtype=f16)
    gather_heads(o, gath, full, world, S, sh.n_heads, hd, eb.EB_F16)
    torch.cuda.synchronize()
    if rank == 0:
        qr = orc.round_f16(orc.rope(q, cos, sin, S, H, hd))
        kr = orc.round_f16(orc.rope(k, cos, sin, S, Hkv, hd))
        want = orc.attn_prefill_part(qr, kr, v, H, Hkv, S, hd, hd ** -0.5, (S - 96, S), (0, H),
                                     nthreads=os.cpu_count() or 8).reshape(S, H, hd)[S - 96:]
        got = full.float().cpu().numpy()[S - 96:]
        ma, rl = orc.max_abs(got, want), orc.rel_l2(got, want)
        print(f"[mgpu] world={world} prefill rows [{S-96},{S}) x {H} heads: max_abs={ma:.2e} "
              f"rel_l2={rl:.2e}", flush=True)
        ok &= ma <= 2e-3 and rl <= 1e-3
    # ---- the same prefill with the gather fused into the kernel (peer TMA
    # stores), and with own-buffer writes + the multicast broadcast
    for mode in ("peer", "multicast"):
        try:
            g = GatheredOutput(S, H, hd, f16, sh, mode=mode)
        except RuntimeError as e:
            if rank == 0:
                print(f"[mgpu] {mode}: {e}", flush=True)
            continue
        g.bufs.fill_(float("nan"))
        g.barrier()
        same = True
        for _ in range(3):  # both buffers, and the first one again
            eb.attention_prefill_gather(desc, layer, S, dev(q[:, sh.h0:sh.h1]),
                                        dev(k[:, sh.kv0:sh.kv1]), dev(v[:, sh.kv0:sh.kv1]), kc,
                                        vc, g.next(), ws)
            g.finish()
            same &= torch.equal(g.full, full)
        torch.cuda.synchronize()
        print(f"[mgpu] rank {rank} gathered output ({mode}) == NCCL gather: {same}", flush=True)
        ok &= same
        del g
    # ---- batched decode: config-5 geometry, 8 sequences, f16 caches
    B, max_seq = 8, 4096
    pos = (np.random.default_rng(12).integers(512, max_seq, size=B) - 1).astype(np.int32)
    kcf = orc.round_f16(rng.standard_normal((B, max_seq, Hkv, hd)).astype(np.float32)).reshape(
        B, max_seq, Hkv, hd)
    vcf = orc.round_f16(rng.standard_normal((B, max_seq, Hkv, hd)).astype(np.float32)).reshape(
        B, max_seq, Hkv, hd)
    qd = orc.round_f16(rng.standard_normal((B, H, hd)).astype(np.float32)).reshape(B, H, hd)
    kd = orc.round_f16(rng.standard_normal((B, Hkv, hd)).astype(np.float32)).reshape(B, Hkv, hd)
    vd = orc.round_f16(rng.standard_normal((B, Hkv, hd)).astype(np.float32)).reshape(B, Hkv, hd)
    cos, sin = eb.rope_tables(max_seq, hd, 5e5)
    desc = eb.make_desc(sh.n_heads, sh.n_kv_heads, hd, max_seq, dtype_qkv=eb.EB_F16,
                        dtype_cache=eb.EB_F16, dtype_out=eb.EB_F16)
    layer = eb.make_layer(rope_cos=torch.from_numpy(cos).cuda(), rope_sin=torch.from_numpy(sin).cuda())
    kcd = dev(kcf[:, :, sh.kv0:sh.kv1])
    vcd = dev(vcf[:, :, sh.kv0:sh.kv1])
    od = torch.empty(B, sh.n_heads, hd, device="cuda", dtype=f16)
    ws = eb.alloc_workspace(eb.attention_decode_workspace_bytes(desc, B, int(pos.max())))
    eb.attention_decode_batched(desc, layer, B, torch.from_numpy(pos).cuda(), int(pos.max()),
                                dev(qd[:, sh.h0:sh.h1]), dev(kd[:, sh.kv0:sh.kv1]),
                                dev(vd[:, sh.kv0:sh.kv1]), kcd, vcd,
                                max_seq * sh.n_kv_heads * hd, od, ws)
    gath = torch.empty(world, B, sh.n_heads, hd, device="cuda", dtype=f16)
    fulld = torch.empty(B, H, hd, device="cuda", dtype=f16)
    gather_heads(od, gath, fulld, world, B, sh.n_heads, hd, eb.EB_F16)
    torch.cuda.synchronize()
    if rank == 0:
        for b in range(B):
            kcf[b, pos[b]] = orc.round_f16(orc.rope(kd[b], cos, sin, 1, Hkv, hd, int(pos[b]))).reshape(Hkv, hd)
            vcf[b, pos[b]] = vd[b]
        qr = np.stack([orc.rope(qd[b], cos, sin, 1, H, hd, int(pos[b])) for b in range(B)])
        want = orc.attn_decode_batched(qr, kcf, vcf, pos, H, Hkv, hd, max_seq,
                                       max_seq * Hkv * hd, hd ** -0.5, nthreads=os.cpu_count() or 8)
        got = fulld.float().cpu().numpy().ravel()
        ma, rl = orc.max_abs(got, want), orc.rel_l2(got, want)
        print(f"[mgpu] world={world} batched decode {B} seqs: max_abs={ma:.2e} rel_l2={rl:.2e}",
              flush=True)
        ok &= ma <= 2e-3 and rl <= 1e-3
    # ---- the same decode with the gather fused into the decode kernel (its
    # output rows stored into every rank's symmetric-memory buffer): by KV-head
    # group (bit-identical to the NCCL gather: same per-rank work), and by
    # sequence only (every rank all heads of a context-balanced bucket of the
    # sequences; checked against the oracle on rank 0)
    for head_groups in (None, 1):
        dsh = decode_shard(H, Hkv, world, rank, pos + 1, head_groups=head_groups)
        seqs = list(dsh.seqs)
        ddesc = eb.make_desc(dsh.n_heads, dsh.n_kv_heads, hd, max_seq, dtype_qkv=eb.EB_F16,
                             dtype_cache=eb.EB_F16, dtype_out=eb.EB_F16)
        g = GatheredOutput(B, H, hd, f16, dsh)
        g.bufs.fill_(float("nan"))
        g.barrier()
        lpos = pos[seqs]
        mp = int(lpos.max()) if seqs else 0
        wsg = eb.alloc_workspace(eb.attention_decode_workspace_bytes(ddesc, max(1, len(seqs)), mp))
        args = (dev(qd[seqs][:, dsh.h0:dsh.h1]), dev(kd[seqs][:, dsh.kv0:dsh.kv1]),
                dev(vd[seqs][:, dsh.kv0:dsh.kv1]),
                dev(kcf[seqs][:, :, dsh.kv0:dsh.kv1]), dev(vcf[seqs][:, :, dsh.kv0:dsh.kv1]))
        sidx = torch.tensor(seqs, dtype=torch.int32, device="cuda")
        same = True
        for _ in range(3):
            eb.attention_decode_batched_gather(ddesc, layer, len(seqs),
                                               torch.from_numpy(np.ascontiguousarray(lpos)).cuda(),
                                               mp, *args, max_seq * dsh.n_kv_heads * hd, g.next(),
                                               sidx, wsg)
            g.finish()
            if head_groups is None:
                same &= torch.equal(g.full, fulld)
        torch.cuda.synchronize()
        if head_groups is None:
            print(f"[mgpu] rank {rank} decode gathered in-kernel == NCCL gather: {same}",
                  flush=True)
            ok &= same
        elif rank == 0:
            got = g.full.float().cpu().numpy().ravel()
            ma, rl = orc.max_abs(got, want), orc.rel_l2(got, want)
            print(f"[mgpu] world={world} decode split by sequence (gathered in-kernel): "
                  f"max_abs={ma:.2e} rel_l2={rl:.2e}", flush=True)
            ok &= ma <= 2e-3 and rl <= 1e-3
        del g
    flag = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(flag)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("[mgpu] PASS" if flag.item() == 0 else "[mgpu] FAIL", flush=True)
    return int(flag.item() != 0)


if __name__ == "__main__":
    sys.exit(main())

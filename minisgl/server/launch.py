"""Process launcher (reference: python/minisgl/server/launch.py:16-113): one scheduler process per
TP rank, one detokenizer (which also tokenizes when ``--num-tokenizer 0``), optional extra
tokenizer processes; waits for all of them to report ready, then serves HTTP or the shell."""

from __future__ import annotations

import multiprocessing as mp
import sys
from dataclasses import replace

from minisgl.utils import init_logger

logger = init_logger(__name__)


def _run_scheduler(args, ack_queue) -> None:
    import torch

    from minisgl.scheduler import Scheduler
    from minisgl.utils.proc import die_with_parent

    die_with_parent()  # a rank never outlives the server process that spawned it

    with torch.inference_mode():
        sched = Scheduler(args)
        sched.sync_all_ranks()
        if args.tp_info.is_primary():
            ack_queue.put("scheduler ready")
        try:
            sched.run_forever()
        except KeyboardInterrupt:
            pass
        finally:
            sched.shutdown()


def launch_server(run_shell: bool = False, argv=None) -> None:
    from minisgl.parallel import DistributedInfo

    from .api_server import run_api_server
    from .args import parse_args

    args = parse_args(sys.argv[1:] if argv is None else argv, run_shell=run_shell)
    logger.info(f"launching: {args.model_path} tp={args.tp_info.size} port={args.server_port}")

    def start_subprocesses() -> None:
        from minisgl.tokenizer.server import tokenize_worker

        ctx = mp.get_context("spawn")
        acks = ctx.Queue()
        world = args.tp_info.size
        for r in range(world):
            ctx.Process(target=_run_scheduler, args=(replace(args, tp_info=DistributedInfo(r, world)), acks),
                        daemon=False, name=f"minisgl-scheduler-{r}").start()
        n_tok = args.num_tokenizer
        ctx.Process(target=tokenize_worker, kwargs=dict(
            tokenizer_path=args.model_path, addr=args.zmq_detokenizer_addr, create=args.tokenizer_create_addr,
            backend_addr=args.zmq_backend_addr, frontend_addr=args.zmq_frontend_addr, local_bs=1,
            tokenizer_id=n_tok, model_source=args.model_source, ack_queue=acks), daemon=True,
            name="minisgl-detokenizer").start()
        for i in range(n_tok):
            ctx.Process(target=tokenize_worker, kwargs=dict(
                tokenizer_path=args.model_path, addr=args.zmq_tokenizer_addr, create=args.tokenizer_create_addr,
                backend_addr=args.zmq_backend_addr, frontend_addr=args.zmq_frontend_addr, local_bs=1,
                tokenizer_id=i, model_source=args.model_source, ack_queue=acks), daemon=True,
                name=f"minisgl-tokenizer-{i}").start()
        for _ in range(n_tok + 2):
            logger.info(acks.get())

    run_api_server(args, start_subprocesses, run_shell=args.shell_mode)


if __name__ == "__main__":
    launch_server()

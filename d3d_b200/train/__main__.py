"""``python -m d3d_b200.train`` — see :mod:`d3d_b200.train.trainer`."""
from .args import parser
from .trainer import train

if __name__ == "__main__":
    import torch.distributed as dist
    try:
        train(parser().parse_args())
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()

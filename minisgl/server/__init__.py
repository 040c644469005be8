from .args import ServerArgs, parse_args
from .launch import launch_server

__all__ = ["ServerArgs", "parse_args", "launch_server"]

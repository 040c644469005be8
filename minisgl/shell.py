"""``python -m minisgl.shell`` forces interactive shell mode (reference: python/minisgl/shell.py)."""

from minisgl.server.launch import launch_server

if __name__ == "__main__":
    launch_server(run_shell=True)

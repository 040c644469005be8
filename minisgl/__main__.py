"""``python -m minisgl`` launches the server (reference: python/minisgl/__main__.py:1-5)."""

from minisgl.server.launch import launch_server

if __name__ == "__main__":
    launch_server()

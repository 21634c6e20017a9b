# Build/run image for modded_nanogpt_b200 on B200 (sm_100a).  The reference ships a CUDA 12.6 / torch-nightly image
# (its `Dockerfile`); this one needs CUDA >= 12.8 for sm_100a and builds the in-tree extension at image build time.
FROM nvidia/cuda:12.9.1-devel-ubuntu24.04
ENV DEBIAN_FRONTEND=noninteractive PYTHONUNBUFFERED=1
RUN apt-get update && apt-get install -y --no-install-recommends python3 python3-pip python3-venv git ninja-build && \
    rm -rf /var/lib/apt/lists/*
RUN python3 -m venv /opt/venv
ENV PATH=/opt/venv/bin:$PATH
RUN pip install --no-cache-dir torch==2.11.0 --index-url https://download.pytorch.org/whl/cu128 && \
    pip install --no-cache-dir numpy pybind11 pytest flash-attn==2.8.3 tiktoken huggingface_hub
WORKDIR /workspace/modded_nanogpt_b200
COPY . .
RUN python build_ext.py
CMD ["bash", "run.sh"]

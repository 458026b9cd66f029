# openmini_v1_b200 serving image for B200 (sm_100a) hosts.
# Build:  docker build -t openmini-b200 .
# Run:    docker run --gpus all -p 8080:8080 -p 50051:50051 openmini-b200 --preset llama7b
FROM nvcr.io/nvidia/pytorch:25.06-py3
ENV PYTHONUNBUFFERED=1 MAX_JOBS=16
WORKDIR /opt/openmini
COPY setup.py pytest.ini ./
COPY csrc ./csrc
COPY include ./include
COPY openmini_v1_b200 ./openmini_v1_b200
COPY config ./config
COPY bench.py __graft_entry__.py ./
RUN pip install --no-cache-dir fastapi uvicorn grpcio protobuf sentencepiece pynvml && \
    python setup.py build_ext --inplace
EXPOSE 8080 50051
HEALTHCHECK --interval=30s --timeout=5s CMD python -c "import urllib.request; urllib.request.urlopen('http://127.0.0.1:8080/health')"
ENTRYPOINT ["python", "-m", "openmini_v1_b200.serve.main", "--config", "config/server.toml"]

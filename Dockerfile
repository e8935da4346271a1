# B200 image for lora_kernel_b200: CUDA 12.9 + PyTorch, extension built for sm_100a.
FROM nvcr.io/nvidia/pytorch:25.06-py3
WORKDIR /opt/lora_kernel_b200
COPY . .
RUN python setup.py build_ext --inplace
ENV PYTHONPATH=/opt/lora_kernel_b200
ENTRYPOINT ["python", "-m", "lora_kernel_b200", "serve"]

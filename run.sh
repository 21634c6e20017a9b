torchrun --standalone --nproc_per_node=8 train_gpt.py

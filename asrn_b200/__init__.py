"""asrn_b200: the ASRN layer forward and its O(1) generation step on NVIDIA B200 (sm_100a).

Drop-in for the reference package's public API on this path (KIROKOWA/ASRN, asrn/__init__.py:60-97):
    ASRNLayer / CapaASRNEstable     the layer (forward on CUDA kernels of libasrn_b200.so)
    create_model / crear_modelo     the language model with ASRN layers after every `largo_cada` local blocks
    generate / escribir             incremental generation with the O(1) per-token writer
    Protecciones / Protections      numeric protections (group A by default)
    guardar / cargar (save / load)  model files in the reference's format (its files load here and ours load there)
"""
from .layer import ASRNLayer, CapaASRNEstable, Protecciones, Protections
from .model import (ASRNModel, BloqueLocal, LocalBlock, ModeloASRN, cargar, create_model, crear_modelo, firmas_de_piezas,
                    guardar, load, save)
from .writer import Escritor, Writer, escribir, generate

__all__ = ['ASRNLayer', 'CapaASRNEstable', 'Protecciones', 'Protections', 'ASRNModel', 'ModeloASRN', 'LocalBlock',
           'BloqueLocal', 'create_model', 'crear_modelo', 'firmas_de_piezas', 'generate', 'escribir', 'Writer',
           'Escritor', 'guardar', 'cargar', 'save', 'load']

__version__ = '0.1'

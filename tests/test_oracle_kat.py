"""Hand-computed known answers at tiny sizes for the oracle (the reference
ships no test vectors for its attention path, so these pin the arithmetic
directly).  Expected values are derived by hand in the comments.

* Gated delta rule (text_modules.rs:365-443, chunked :189-363), H=1, d_k=d_v=2,
  T=2.  Step 1: q=[1,0], k=[0,2] -> k^=[0,1]; v=[4,6], g=0, beta=0.5; S=0, so
  delta=(v-0)*0.5=[2,3], S=[[0,0],[2,3]], o=S^T q^=[0,0].  Step 2: q=[0,3] ->
  q^=[0,1]/sqrt2 (scale 2^-1/2), k=[1,1] -> k^=[1,1]/sqrt2, v=[1,1], g=ln(1/2),
  beta=1; S*1/2=[[0,0],[1,1.5]], m=S^T k^=[1,1.5]/sqrt2, delta=v-m, S+=k^ delta^T
  = [[0.20710678,-0.04289322],[1.20710678,1.45710678]], o=S^T q^=S[1]/sqrt2
  = [0.85355339,1.03033009].
* GQA decode (:842-944), d=4, one q and one kv head, no RoPE: q=[1,1,1,1]
  (RMSNorm leaves it), cached key [2,0,0,0], new key [0,2,0,0] (RMSNorm: mean
  square 1, unchanged); both scores are 2/sqrt(4)=1, so the softmax is 1/2,1/2,
  attention = mean([1,2,3,4],[5,6,7,8]) = [3,4,5,6], gate 0 -> sigmoid 1/2,
  out = [1.5,2,2.5,3].
* RoPE at position 0 is the identity (cos 1, sin 0).
Tolerance 1e-5 (the l2norm / RMSNorm eps of 1e-6 inside the square roots).
"""
import math

import numpy as np

import oracle


def test_gated_delta_rule_two_steps():
    f = np.float32
    q = np.array([[[[1, 0]]], [[[0, 3]]]], f).reshape(1, 2, 1, 2)
    k = np.array([[[[0, 2]]], [[[1, 1]]]], f).reshape(1, 2, 1, 2)
    v = np.array([[[[4, 6]]], [[[1, 1]]]], f).reshape(1, 2, 1, 2)
    g = np.array([0.0, math.log(0.5)], f).reshape(1, 2, 1)
    beta = np.array([0.5, 1.0], f).reshape(1, 2, 1)
    S0 = np.zeros((1, 1, 2, 2), f)
    out_exp = np.array([[0, 0], [0.85355339, 1.03033009]], f)
    S_exp = np.array([[0.20710678, -0.04289322], [1.20710678, 1.45710678]], f)
    for fn in (lambda: oracle.recurrent_gdr(q, k, v, g, beta, S0),
               lambda: oracle.chunk_gdr(q, k, v, g, beta, S0, chunk=2),
               lambda: oracle.chunk_gdr(q, k, v, g, beta, S0, chunk=64)):
        out, S = fn()
        np.testing.assert_allclose(out.reshape(2, 2), out_exp, atol=1e-5)
        np.testing.assert_allclose(S.reshape(2, 2), S_exp, atol=1e-5)


def test_gqa_equal_scores_average_the_values():
    f = np.float32
    q_gate = np.array([[[1, 1, 1, 1, 0, 0, 0, 0]]], f)          # [B=1, Hq=1, 2D]: q | gate
    k_new = np.array([[[0, 2, 0, 0]]], f)
    v_new = np.array([[[5, 6, 7, 8]]], f)
    kc = np.zeros((1, 1, 4, 4), f)
    vc = np.zeros((1, 1, 4, 4), f)
    kc[0, 0, 0] = [2, 0, 0, 0]
    vc[0, 0, 0] = [1, 2, 3, 4]
    w0 = np.zeros(4, f)
    cos, sin = np.ones((1, 4), f), np.zeros((1, 4), f)
    out, kc2, vc2, lens = oracle.gqa_decode(q_gate, k_new, v_new, w0, w0, cos, sin, kc, vc, np.array([1], np.int32),
                                            rot=0)
    np.testing.assert_allclose(out.reshape(4), [1.5, 2.0, 2.5, 3.0], atol=1e-5)
    assert int(lens[0]) == 2
    np.testing.assert_allclose(kc2[0, 0, 1], [0, 2, 0, 0], atol=1e-5)
    np.testing.assert_array_equal(vc2[0, 0, 1], [5, 6, 7, 8])


def test_rope_position_zero_is_identity():
    cos, sin = oracle.rope_tables(np.array([0], np.int64), rot=64, theta=1e7)
    assert np.all(cos == 1.0) and np.all(sin == 0.0)

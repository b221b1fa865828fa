"""A Python model of the GPU sampler's pass algorithm (csrc/sample.cu): FP64
running sums computed per binade as compositions of parity-dependent integer
maps, one-thread handling of groups that may cross a binade or hold the
stop, closed-form jumps over steady stretches. Used by the CPU tests to check
the algorithm against the sequential oracle (small chunks exercise many
chunk boundaries and events)."""
import math

SAT = 1 << 60
T52, T53 = 1 << 52, 1 << 53
ADD, TOPP, SUB = 0, 1, 2


def _sat(v):
    return max(-SAT, min(SAT, v))


def _mul_sat(n, d):
    return SAT if n * d > SAT else n * d


def decode(t):
    if not (t > 0.0) or math.isinf(t) or t < 2.2250738585072014e-308:
        return None
    fm, ex = math.frexp(t)
    return int(fm * (1 << 53)), ex - 53


def classify(p, e):
    x = math.ldexp(p, -e)
    if not (x < 2.0 ** 62):
        return 0, 3
    fm = math.floor(x)
    f = x - fm
    return int(fm), (0 if f < 0.5 else (1 if f > 0.5 else 2))


def compose(a, b):
    return (_sat(a[0] + (b[1] if a[0] & 1 else b[0])),
            _sat(a[1] + (b[1] if (a[1] + 1) & 1 else b[0])))


def group_elem(m, cls, c, sub):
    if cls == 3:
        r = (SAT, SAT)
    elif cls == 2:
        rest = _mul_sat(c - 1, m + (m & 1))
        r = (_sat(rest + (m + 1 if m & 1 else m)), _sat(rest + (m if m & 1 else m + 1)))
    else:
        r = (_mul_sat(c, m + cls),) * 2
    return (-r[0], -r[1]) if sub else r


def apply(T, el):
    return T + (el[1] if T & 1 else el[0])


def run_steps(t, p, count, mode, thr):
    """One thread: real FP64 steps where the binade may change or a stop may
    come, closed-form jumps otherwise. Returns (stopped, pos, t)."""
    done = 0
    while done < count:
        if mode == SUB:
            if t <= p:
                return True, done, t - p
            t = t - p
        else:
            t = t + p
            if mode == TOPP and t >= thr:
                return True, done, t
        done += 1
        if done == count:
            break
        d_ = decode(t)
        if d_ is None:
            continue
        T, e = d_
        m, cls = classify(p, e)
        if cls == 3 or (cls == 2 and T & 1):
            continue
        d = m + (m & 1) if cls == 2 else m + cls
        rem = count - done
        if mode == SUB:
            room = T - (T52 + 1)
            if room < 0:
                continue
            n = rem if d == 0 else min(rem, room // d)
            if n <= 0:
                continue
            T -= n * d
        else:
            room = (T53 - 1) - T - m
            if room < 0:
                continue
            n = rem if d == 0 else min(rem, room // d + 1)
            if mode == TOPP and d > 0:
                thr_t = math.ldexp(thr, -e)
                if thr_t < 2.0 ** 62:
                    jt = (math.ceil(thr_t) - T + d - 1) // d
                    if jt <= n:
                        return True, done + jt - 1, math.ldexp(float(T + jt * d), e)
            T += n * d
        t = math.ldexp(float(T), e)
        done += n
    return False, count, t


def run_pass(mode, t, counts, weights, thr, chunk=8):
    """The block's pass: scan a chunk in the current binade, hand the first
    unsafe group to one thread, resume behind it. Returns (t, stop)."""
    sub = mode == SUB
    g = 0
    n = len(counts)
    while g < n:
        d_ = decode(t)
        if d_ is None:
            stop, pos, t = run_steps(t, weights[g], counts[g], mode, thr)
            if stop:
                return t, (g, pos)
            g += 1
            continue
        T0, e = d_
        end = min(n, g + chunk)
        T, bad = T0, None
        for j in range(g, end):  # sequential composition == the block scan's prefix
            m, cls = classify(weights[j], e)
            tend = apply(T, group_elem(m, cls, counts[j], sub))
            if cls == 3:
                ok = False
            elif sub:
                ok = tend >= T52 + 1
            else:
                ok = tend + m <= T53 - 1 and (mode != TOPP or math.ldexp(float(tend), e) < thr)
            if not ok:
                bad = (j, T)
                break
            T = tend
        if bad is None:
            t = math.ldexp(float(T), e)
            g = end
            continue
        j, Tb = bad
        stop, pos, t = run_steps(math.ldexp(float(Tb), e), weights[j], counts[j], mode, thr)
        if stop:
            return t, (j, pos)
        g = j + 1
    return t, None


def sample_model(order_keys, weights_of_key, top_p, u):
    """Groups (key, count) in descending order, then total, top-p and walk as
    the kernel runs them; u = the XorShift64 draw in [0, 1). Returns
    (group index, position) of the chosen candidate or None."""
    keys = sorted(set(order_keys), reverse=True)
    counts = [order_keys.count(k) for k in keys]
    weights = [weights_of_key(k) for k in keys]
    total, _ = run_pass(ADD, 0.0, counts, weights, 0.0)
    if top_p < 1.0:
        t, stop = run_pass(TOPP, 0.0, counts, weights, total * top_p)
        counts = counts[:stop[0] + 1]
        counts[-1] = stop[1] + 1
        weights = weights[:stop[0] + 1]
        total = t
    _, stop = run_pass(SUB, u * total, counts, weights, 0.0)
    return keys, stop

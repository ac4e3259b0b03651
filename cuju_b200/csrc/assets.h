// cuju-b200 host: the read-only inputs of a batch.
//   - `animations.bin` (CUJANIM1): animations, node key frames, football keys, positions,
//     quadrants (cuju include/cuju/animation/animation_data.h:170-300), plus what is derived
//     from them once at load: the interpolation table (keyframes.h:132), the values parsed from
//     each animation's text variables (animation_derived.h:105), the per-animation selection
//     terms and the function-type index (simulation/select_animation.h:484-566), the smoothed
//     movement per frame and the camera weights (batch/tables.h:24-90).
//   - asset bundles (CUJASSET1): scenario, agent counts and four variants of static data, reset
//     state and skeletons (batch/batch_core.h:686-752), with the agent setup of
//     batch/agent_setup.h:20-160.
// Every derived value is computed with the same host/device functions the simulation uses, so a
// table read equals the computation bit for bit.
#pragma once

#include <algorithm>
#include <fstream>
#include <map>
#include <memory>
#include <sstream>

#include "codec.h"
#include "env.cuh"

namespace cb {
namespace host {

inline std::string read_file(const std::string &path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

struct Reader {
    const std::string &b;
    const char *what;
    size_t off;
    template <class T>
    T get() {
        if (off + sizeof(T) > b.size()) throw std::runtime_error(std::string(what) + " end early");
        T v;
        memcpy(&v, b.data() + off, sizeof(T));
        off += sizeof(T);
        return v;
    }
    std::string str() {
        int32_t n = get<int32_t>();
        if (n < 0 || off + (size_t)n > b.size()) throw std::runtime_error(std::string("a string of ") + what + " runs past their end");
        std::string s = b.substr(off, (size_t)n);
        off += (size_t)n;
        return s;
    }
    bool end() const { return off == b.size(); }
};

inline int32_t intern_state_string(const std::string &t) {
    static const char *const known[] = {"", "lay_back", "lay_front", "left_elbow", "right_elbow"};
    for (int32_t i = 0; i < 5; i++)
        if (t == known[i]) return i;
    throw std::runtime_error("expected a known state string in the animation tables, found `" + t + "`");
}
inline int body_part_from_string(const std::string &p) {
    static const char *names[] = {"middle", "neck", "left_thigh", "right_thigh", "left_knee", "right_knee",
                                  "left_ankle", "right_ankle", "left_shoulder", "right_shoulder",
                                  "left_elbow", "right_elbow", "body", "player"};
    for (int i = 0; i < 14; i++)
        if (p == names[i]) return i;
    return -1;
}
inline std::vector<std::string> tokenize(const std::string &t, const std::string &d) {
    std::vector<std::string> out;
    std::string::size_type s = t.find_first_not_of(d, 0), e = t.find_first_of(d, s);
    while (std::string::npos != e || std::string::npos != s) {
        out.push_back(t.substr(s, e - s));
        s = t.find_first_not_of(d, e);
        e = t.find_first_of(d, s);
    }
    return out;
}
// GRF's GetVectorFromString: comma-separated, parsed with the C library's atof.
inline Vec3 vector_from_string(const std::string &t) {
    if (t.empty()) return Vec3(0.0f);
    std::vector<std::string> tk = tokenize(t, ",");
    Vec3 r;
    r.c[0] = (float)atof(tk.at(0).c_str());
    if (tk.size() > 1) r.c[1] = (float)atof(tk.at(1).c_str());
    if (tk.size() > 2) r.c[2] = (float)atof(tk.at(2).c_str());
    return r;
}

// Host copies of every table in AnimTables, plus the text variables.
struct AnimStore {
    std::vector<Anim> anims;
    std::vector<AnimDerived> derived;
    std::vector<NodeAnim> nodes;
    std::vector<KeyFrame> keys;
    std::vector<InterpEntry> interp;
    std::vector<FootballKey> football;
    std::vector<Vec3> positions;
    std::vector<Quadrant> quadrants;
    std::vector<int16_t> functionAnims;
    std::vector<int32_t> functionOffsets;
    std::vector<Vec3> smoothed;
    std::vector<float> cameraWeights;
    std::vector<std::map<std::string, std::string>> vars;
    Radian maxIn, maxOut;
    std::string var(size_t i, const std::string &k) const {
        auto e = vars[i].find(k);
        return e == vars[i].end() ? std::string() : e->second;
    }
};

inline void derive(AnimStore &st);

inline std::unique_ptr<AnimStore> parse_animations(const std::string &bytes) {
    if (bytes.compare(0, 8, "CUJANIM1") != 0) throw std::runtime_error("expected the animation tables, found another file");
    Reader r{bytes, "the animation tables", 8};
    auto st = std::make_unique<AnimStore>();
    const int32_t n = r.get<int32_t>();
    if (n < 0 || n > 32767) throw std::runtime_error("the animation tables hold too many animations");
    st->anims.resize(n);
    st->vars.resize(n);
    for (int32_t i = 0; i < n; i++) {
        Anim &a = st->anims[i];
        memset(&a, 0, sizeof(a));
        r.str();  // name
        a.frameCount = r.get<int32_t>();
        a.currentFoot = r.get<int32_t>();
        a.animationType = r.get<int32_t>();
        a.translation = r.get<Vec3>();
        a.incomingMovement = r.get<Vec3>();
        a.incomingVelocity = r.get<float>();
        a.outgoingMovement = r.get<Vec3>();
        a.outgoingDirection = r.get<Vec3>();
        a.incomingBodyDirection = r.get<Vec3>();
        a.outgoingBodyDirection = r.get<Vec3>();
        a.outgoingVelocity = r.get<float>();
        a.outgoingAngle = r.get<Radian>();
        a.incomingBodyAngle = r.get<Radian>();
        a.outgoingBodyAngle = r.get<Radian>();
        a.outgoingFoot = r.get<int32_t>();
        a.idleLevel = r.get<float>();
        a.quadrantID = r.get<int32_t>();
        a.specialVar1 = r.get<float>();
        a.specialVar2 = r.get<float>();
        a.lastDitch = r.get<uint8_t>() != 0;
        a.baseAnimation = r.get<uint8_t>() != 0;
        a.outgoingSpecialState = intern_state_string(r.str());
        a.incomingRetainState = intern_state_string(r.str());
        a.incomingSpecialState = intern_state_string(r.str());
        const int32_t nv = r.get<int32_t>();
        for (int v = 0; v < nv; v++) {
            std::string k = r.str();
            st->vars[i][k] = r.str();
        }
        const int32_t nn = r.get<int32_t>();
        if (nn < 0 || nn > kBodyParts) throw std::runtime_error("an animation holds too many nodes");
        a.firstNode = (int32_t)st->nodes.size();
        a.nodeCount = nn;
        for (int k = 0; k < nn; k++) {
            NodeAnim na;
            memset(&na, 0, sizeof(na));
            na.bodyPart = r.get<int32_t>();
            if (na.bodyPart < 0 || na.bodyPart >= kBodyParts)
                throw std::runtime_error("expected body parts from 0 to 13 in the animation tables");
            for (int32_t e = a.firstNode; e < (int32_t)st->nodes.size(); e++)
                if (st->nodes[e].bodyPart == na.bodyPart)
                    throw std::runtime_error("the animation tables repeat a body part within an animation");
            const int32_t nk = r.get<int32_t>();
            if (nk < 1) throw std::runtime_error("an animation node without keys");
            na.firstKey = (int32_t)st->keys.size();
            na.keyCount = nk;
            for (int j = 0; j < nk; j++) {
                KeyFrame kf;
                kf.frame = r.get<int32_t>();
                kf.orientation = r.get<Quat>();
                kf.position = r.get<Vec3>();
                st->keys.push_back(kf);
            }
            st->nodes.push_back(na);
        }
        a.hasFootball = r.get<int32_t>() != 0;
        a.firstFootball = (int32_t)st->football.size();
        a.footballCount = 0;
        if (a.hasFootball) {
            const int32_t nf = r.get<int32_t>();
            a.footballCount = nf;
            for (int j = 0; j < nf; j++) {
                FootballKey fk;
                fk.frame = r.get<int32_t>();
                fk.orientation = r.get<Quat>();
                fk.position = r.get<Vec3>();
                fk.power = r.get<float>();
                st->football.push_back(fk);
            }
        }
        const int32_t np = r.get<int32_t>();
        a.hasPositions = np >= 0;
        a.firstPosition = (int32_t)st->positions.size();
        a.positionCount = np > 0 ? np : 0;
        if (a.positionCount > kAnimPositions || a.frameCount > kAnimPositions)
            throw std::runtime_error("expected animations of at most 320 frames");
        for (int j = 0; j < np; j++) st->positions.push_back(r.get<Vec3>());
    }
    const int32_t nq = r.get<int32_t>();
    st->quadrants.resize(nq);
    for (Quadrant &q : st->quadrants) {
        q.id = r.get<int32_t>();
        q.position = r.get<Vec3>();
        q.velocity = r.get<int32_t>();
        q.angle = r.get<Radian>();
    }
    st->maxIn = r.get<Radian>();
    st->maxOut = r.get<Radian>();
    if (!r.end()) throw std::runtime_error("the animation tables hold bytes after their end");
    derive(*st);
    return st;
}

inline void derive(AnimStore &st) {
    const int n = (int)st.anims.size();
    // Interpolation: frames 0..frameCount+1 of every node (keyframes.h:132).
    size_t total = 0;
    for (const Anim &a : st.anims) total += (size_t)a.nodeCount * (a.frameCount + 2);
    st.interp.assign(total, InterpEntry{});
    size_t off = 0;
    for (const Anim &a : st.anims) {
        const int frames = a.frameCount + 2;
        for (int k = 0; k < a.nodeCount; k++) {
            NodeAnim &na = st.nodes[a.firstNode + k];
            for (int f = 0; f < frames; f++) {
                InterpEntry &e = st.interp[off + f];
                interpolate_keys(a, st.keys.data() + na.firstKey, na.keyCount, f, e.orientation, e.position);
                float x, y;
                e.orientation.angles(x, y, e.angleZ);
            }
            na.interpOffset = (int32_t)off;
            na.interpFrames = frames;
            off += frames;
        }
    }
    // Text variables (animation_derived.h:105, DeriveAll), parsed with the C library.
    st.derived.assign(n, AnimDerived{});
    for (int i = 0; i < n; i++) {
        AnimDerived &d = st.derived[i];
        memset(&d, 0, sizeof(d));
        const Anim &a = st.anims[i];
        auto V = [&](const char *k) { return st.var(i, k); };
        d.priorityAbsolute = fabs(atof(V("priority").c_str()));
        d.touchFrame = atoi(V("touchframe").c_str());
        d.animDifficultyFactor = (float)atof(V("animdifficultyfactor").c_str());
        d.tripTypeIsOne = V("triptype") == "1";
        d.tripTypeRounded = (int)round(atof(V("triptype").c_str()));
        d.bumpDirection = vector_from_string(V("bumpdirection"));
        d.incomingBallDirection = vector_from_string(V("incomingballdirection"));
        d.ballDirection = vector_from_string(V("balldirection"));
        d.incomingMaxDeviation = (float)fabs(atof(V("incomingballdirection_maxdeviation").c_str()) * kPi);
        d.outgoingMaxDeviation = (float)fabs(atof(V("outgoingballdirection_maxdeviation").c_str()) * kPi);
        const std::string ors = V("outgoing_retain_state"), irs = V("incoming_retain_state");
        d.outgoingRetainRawValue = intern_state_string(ors);
        d.outgoingRetainRaw = !ors.empty();
        d.incomingRetainRawValue = intern_state_string(irs);
        d.outgoingRetainBodyPart = ors.empty() ? -1 : body_part_from_string(ors);
        d.incomingRetainBodyPart = irs.empty() ? -1 : body_part_from_string(irs);
        const std::string ff = V("forcedfoot");
        d.forcedFootWhich = ff == "strong" ? 1 : ff == "weak" ? 2 : 0;
        d.touchFootLeft = V("touchfoot") == "left";
        const std::string tb = V("touch_bodypart");
        d.touchType = (tb.find("foot") != std::string::npos || tb.find("lowerleg") != std::string::npos) ? 0 : 1;
        d.touchMaxPowerFactor = (float)atof(V("touch_maxpowerfactor").c_str());
        d.touchDifficultyFactor = (float)atof(V("touch_difficultyfactor").c_str());
        d.crudeOutDirectionRotated = rot2d(a.outgoingDirection, a.outgoingBodyAngle.value());
        d.crudeTurnAngle = angle2d_to(d.crudeOutDirectionRotated, a.incomingBodyDirection);
        d.crudeInBodyFixAbsolute = fabsf(wrap_range(-kPi, kPi, angle2d(a.incomingBodyDirection) + 0.5f * kPi));
        d.crudeOutBodyDirection = rot2d(Vec3(0, -1, 0), a.outgoingBodyAngle.value() + a.outgoingAngle.value());
        d.crudeInBallNonzero = d.incomingBallDirection.length() != 0.0f;
        d.crudeInBallAdapted = d.incomingBallDirection;
        d.crudeInBallAdapted.c[2] *= 0.4f;
        if (d.crudeInBallNonzero) d.crudeInBallAdapted.normalize();
        d.crudeBallDirectionNormalized = d.ballDirection;
        d.crudeBallDirectionNormalized.normalize(Vec3(0));
        // Selection terms (select_animation.h:484, MakeSelectionRecord).
        for (int k = 0; k < 6; k++) d.incomingBodyAngles[k] = angle2d_to(a.incomingBodyDirection, allowed_body_dir(k));
        d.bodyTurnAngle = angle2d_to(a.incomingBodyDirection, d.crudeOutBodyDirection);
        d.incomingBodyIndex = force_allowed_body_index(a.incomingBodyDirection);
        d.preferredOutgoingDirection = force_preferred_vector(a.outgoingDirection);
        d.preferredOutgoingMovement = d.preferredOutgoingDirection * range_velocity(a.outgoingVelocity);
        d.preferredOutgoingAngle = force_preferred_angle(a.outgoingAngle.value());
        d.lookAngle = force_allowed_body_angle_value(a.outgoingBodyAngle.value()) + d.preferredOutgoingAngle;
        d.smoothedMovementOffset = a.positionCount >= 2 ? a.firstPosition : -1;
        const Vec3 &bd = d.crudeBallDirectionNormalized;
        d.ballDirectionFinite = std::isfinite(bd.c[0]) && std::isfinite(bd.c[1]) && std::isfinite(bd.c[2]);
    }
    // Smoothed movement, parallel to `positions`.
    st.smoothed.assign(st.positions.size(), Vec3(0));
    for (int i = 0; i < n; i++) {
        const Anim &a = st.anims[i];
        if (st.derived[i].smoothedMovementOffset < 0) continue;
        for (uint32_t f = 0; f < (uint32_t)a.positionCount; f++)
            st.smoothed[a.firstPosition + f] =
                movement_at_frame(st.positions.data() + a.firstPosition, a.positionCount, f, 1);
    }
    // Function-type index: animations per function type, in increasing order.
    st.functionAnims.clear();
    st.functionOffsets.assign(kFunctionTypeSlots + 1, 0);
    for (int ft = 0; ft < kFunctionTypeSlots; ft++) {
        st.functionOffsets[ft] = (int32_t)st.functionAnims.size();
        for (int i = 0; i < n; i++)
            if (check_function_type(st.anims[i].animationType, ft)) st.functionAnims.push_back((int16_t)i);
    }
    st.functionOffsets[kFunctionTypeSlots] = (int32_t)st.functionAnims.size();
    // Camera weights: for every position count n, the weights of entries 0..n-1.
    st.cameraWeights.assign(kCamPositions * (kCamPositions + 1) / 2, 0.0f);
    for (int c = 1; c <= (int)kCamPositions; c++)
        for (int i = 0; i < c; i++) st.cameraWeights[c * (c - 1) / 2 + i] = camera_weight(i, c);
}

inline std::vector<Skeleton> parse_skeletons(const std::string &bytes) {
    if (bytes.compare(0, 7, "CUJHUM1") != 0) throw std::runtime_error("expected the skeletons of a bundle, found other bytes");
    Reader r{bytes, "the skeletons", 7};
    const int32_t n = r.get<int32_t>();
    if (n < 0 || n > kStaticEntries) throw std::runtime_error("a bundle holds too many skeletons");
    std::vector<Skeleton> out(n);
    for (Skeleton &sk : out) {
        memset(&sk, 0, sizeof(sk));
        for (int b = 0; b < kBodyParts; b++) sk.nodeMap[b] = r.get<int32_t>();
        sk.nodeCount = r.get<int32_t>();
        if (sk.nodeCount < 0 || sk.nodeCount > kNodes) throw std::runtime_error("a skeleton holds too many nodes");
        for (int k = 0; k < sk.nodeCount; k++) {
            SkelNode &nd = sk.nodes[k];
            r.str();
            nd.parent = r.get<int32_t>();
            nd.localMode = r.get<int32_t>();
            nd.position = r.get<Vec3>();
            nd.rotation = r.get<Quat>();
            nd.scale = r.get<Vec3>();
            nd.geometryCount = r.get<int32_t>();
            if (nd.geometryCount < 0 || nd.geometryCount > 2) throw std::runtime_error("a skeleton node holds too many geometries");
            for (int g = 0; g < nd.geometryCount; g++) {
                SkelGeometry &ge = nd.geometries[g];
                const std::string name = r.str();
                ge.footOrLowerLeg = name == "left_foot" || name == "right_foot" || name == "left_lowerleg" ||
                                    name == "right_lowerleg";
                ge.localMode = r.get<int32_t>();
                ge.position = r.get<Vec3>();
                ge.rotation = r.get<Quat>();
                ge.scale = r.get<Vec3>();
                ge.bbMin = r.get<Vec3>();
                ge.bbMax = r.get<Vec3>();
            }
        }
        for (int b = 0; b < kBodyParts; b++)
            if (sk.nodeMap[b] < 0 || sk.nodeMap[b] >= (sk.nodeCount > 0 ? sk.nodeCount : 1))
                throw std::runtime_error("a skeleton maps a body part to no node");
    }
    if (!r.end()) throw std::runtime_error("the skeletons hold bytes after their end");
    return out;
}

// The static data blob: a count, the PlayerData of each entry, then `FORM` (each player's
// formation), `MDUR` (match duration factor) and `SIDS` (stable IDs) (static_data.h:70).
inline StaticData parse_static(const std::string &b) {
    StaticData sd;
    memset(&sd, 0, sizeof(sd));
    sd.matchDurationFactor = 0x1.c5d638p-5f;
    if (b.size() < 4) throw std::runtime_error("static data: too short");
    memcpy(&sd.count, b.data(), 4);
    size_t off = 4 + (size_t)(sd.count > 0 ? sd.count : 0) * sizeof(PlayerData);
    if (sd.count < 3 || sd.count > kStaticEntries || b.size() < off) throw std::runtime_error("static data: bad size");
    memcpy(sd.data, b.data() + 4, sd.count * sizeof(PlayerData));
    const int pc = sd.count - 3;
    const size_t eb = 4 + 12 + 12 + 1 + 1;
    if (b.compare(off, 4, "FORM") != 0 || b.size() < off + 4 + pc * eb)
        throw std::runtime_error("static data: missing or bad formation section");
    off += 4;
    for (int p = 0; p < pc; p++) {
        StaticFormation &f = sd.formation[p];
        memcpy(&f.role, &b[off], 4);
        memcpy(&f.position, &b[off + 4], 12);
        memcpy(&f.startPosition, &b[off + 16], 12);
        f.lazy = b[off + 28] != 0;
        f.controllable = b[off + 29] != 0;
        off += eb;
    }
    if (b.compare(off, 4, "MDUR") != 0 || b.size() < off + 8) throw std::runtime_error("static data: missing or bad match duration section");
    memcpy(&sd.matchDurationFactor, &b[off + 4], 4);
    off += 8;
    if (b.compare(off, 4, "SIDS") != 0 || b.size() != off + 4 + (size_t)sd.count * 4)
        throw std::runtime_error("static data: missing or bad stable ID section");
    memcpy(sd.stableID, &b[off + 4], (size_t)sd.count * 4);
    return sd;
}

// ---------------------------------------------------------------------------------------------
// Agents (agent_setup.h). A reset disables and releases every keyboard and sets its mirror (-1
// for a right agent); the state stores direction times mirror, so a right release is -0.
inline Keyboard reset_keyboard(float mirror) {
    Keyboard k;
    memset(&k, 0, sizeof(k));
    k.mirror = mirror;
    k.direction = Vec3(0, 0, 0) * mirror;
    k.disabled = true;
    return k;
}
inline HumanGamer new_gamer(int slot, int keyboardIndex, float mirror) {
    HumanGamer g;
    memset(&g, 0, sizeof(g));
    g.selectedPlayer = -1;
    g.team = slot;
    g.keyboardIndex = keyboardIndex;
    ControllerState &b = g.controller.base;
    b.player = -1;
    b.team = -1;
    b.opponentTeam = -1;
    b.opponentPlayer = -1;
    b.inputDirection = Vec3(0, -1, 0);
    b.inputVelocityFloat = 0;
    b.timeNeeded_ms = 0;
    b.mentalImageTime = 0;
    b.hasPossession = b.hasUniquePossession = b.teamHasPossession = b.teamHasUniquePossession =
        b.oppTeamHasPossession = b.oppTeamHasUniquePossession = b.hasBestPossession = b.teamHasBestPossession =
            b.hasBestChanceOfPossession = false;
    b.possessionAmount = 0.9f;
    b.teamPossessionAmount = 1.0f;
    b.oppTimeNeededToGetToBall = 100;
    // The human controller's reset overrides these of the player controller's.
    b.lastSwitchTime_ms = (uint64_t)(int64_t)-10000;
    b.lastSwitchTimeDuration_ms = 300;
    b.fadingTeamPossessionAmount = 1.0f;
    HumanControllerState &c = g.controller;
    c.keyboard = reset_keyboard(mirror);
    c.actionMode = 0;
    c.actionButton = kBtnShortPass;
    c.actionBufferTime_ms = 0;
    c.gauge_ms = 0;
    c.previousDirection = Vec3(0, -1, 0);
    c.steadyDirection = Vec3(0, -1, 0);
    c.lastSteadyDirectionSnapshotTime_ms = 0;
    return g;
}
inline void check_agents(const Scenario &sc, int l, int r, const std::string &bundle) {
    auto chk = [&](const char *side, int a, int n) {
        if (a < 0 || a > n)
            throw std::invalid_argument("expected from 0 to " + std::to_string(n) + " " + side +
                                        " agents, the players of the " + side + " team of " + bundle +
                                        ", found " + std::to_string(a));
    };
    chk("left", l, sc.leftTeamSize);
    chk("right", r, sc.rightTeamSize);
    if (l + r > kMatchKeyboards)
        throw std::invalid_argument("expected at most 22 agents in " + bundle + ", found " + std::to_string(l + r));
}
// Gives a template (rest frame) `l` and `r` agents as GRF's reset does: left agent i gets
// keyboard i and right agent i keyboard 11 + i (agent_setup.h:103, SetupAgents).
inline void setup_agents(Match &w, const StaticData &sd, int l, int r, const std::string &bundle) {
    Scenario &sc = w.scenario;
    MatchState &m = w.m;
    check_agents(sc, l, r, bundle);
    sc.leftAgents = 0;
    sc.rightAgents = 0;
    for (Team &t : m.teams) {
        t.gamers.count = 0;
        t.switchPriority.count = 0;
        t.mainSelectedPlayer = -1;
    }
    for (int p = 0; p < m.playerCount; p++) m.players[p].base.externalController = -1;
    m.freeControllerCount = kMatchKeyboards;
    for (int k = 0; k < kMatchKeyboards; k++) m.freeControllers[k] = reset_keyboard(1.0f);
    sc.leftAgents = l;
    sc.rightAgents = r;
    const int agents[2] = {l, r};
    for (int t = 0; t < 2; t++) {
        Team &team = team_by_id(w, t);
        team.gamers.count = agents[t];
        team.switchPriority.count = agents[t];
        for (int g = 0; g < agents[t]; g++) team.switchPriority.el[g] = g;
    }
    for (int t = 0; t < 2; t++) {
        // Both teams still face side -1 at the controller setup, so the right keyboards mirror.
        const float mirror = t == 1 && team_side(w, 1) == -1 ? -1.0f : 1.0f;
        for (int g = 0; g < agents[t]; g++) {
            const int gi = global_gamer(w, t, g);
            HumanGamer &h = gamer_global(w, gi);
            h = new_gamer(team_slot(w, t), g + (t ? kTeamControllers : 0), mirror);
            m.secondKeyboardCopies[gi] = h.controller.keyboard;
        }
    }
    m.freeControllerCount = kMatchKeyboards - l - r;
    // The active controllable players closest to the ball (origin; players at their formation
    // spots), ties in state order; the closest is the main selected player, and by stable ID the
    // players go to the gamers in order.
    Context ctx;
    memset(&ctx, 0, sizeof(ctx));
    ctx.staticData = &sd;
    int32_t status = 0;
    Sim s{w, ctx, nullptr, &status};
    for (int t = 0; t < 2; t++) {
        if (agents[t] == 0) continue;
        const Vec3 ball = ball_predict(m.ball, 0).flat();
        PlayerList ps;
        closest_players(ps, s, t, ball, true, (unsigned int)agents[t], true);
        if (ps.count == 0) continue;
        team_by_id(w, t).mainSelectedPlayer = ps[0];
        std::sort(ps.el, ps.el + ps.count, [&](int a, int b) { return sd.stableID[a] < sd.stableID[b]; });
        for (int g = 0; g < ps.count; g++) gamer_set_selected(w, global_gamer(w, t, g), ps[g]);
    }
}

// One scenario variant of a bundle: the template is the world right after a GRF reset, in the
// rest frame.
struct AssetVariant {
    int reverse = 0, parity = 0;
    int freeControllerCount = 0;
    StaticData staticData;
    std::unique_ptr<Match> world;
    std::string scenario;  // scenario bytes without seed and difficulties
    std::vector<Skeleton> skeletons;
};
struct Assets {
    std::string scenario;
    int leftAgents = 0, rightAgents = 0;
    AssetVariant variants[4];  // reverse * 2 + parity
};

// The scenario bytes of a world without the per-episode seed and the batch-set difficulties.
inline std::string save_scenario(const Match &w) {
    Scenario sc = w.scenario;
    sc.gameEngineRandomSeed = 0;
    sc.leftTeamDifficulty = 0;
    sc.rightTeamDifficulty = 0;
    Archive a{false, std::string()};
    sc.io(a);
    return a.bytes;
}

// `CUJASSET1`, the scenario name, the two agent counts, the variant count (4), then per variant
// its reverse flag, parity, static data, reset state and skeletons; integers int32, blocks
// length-prefixed. -1 keeps the bundle's agent count (batch_core.h:689, LoadAssets).
inline Assets load_assets(const std::string &path, int leftAgents = -1, int rightAgents = -1) {
    const std::string bytes = read_file(path);
    if (bytes.compare(0, 9, "CUJASSET1") != 0) throw std::runtime_error("not an asset bundle: " + path);
    Reader r{bytes, "the asset bundle", 9};
    auto blob = [&]() {
        const uint32_t n = (uint32_t)r.get<int32_t>();
        if (r.off + n > bytes.size()) throw std::runtime_error("asset bundle truncated: " + path);
        std::string b = bytes.substr(r.off, n);
        r.off += n;
        return b;
    };
    Assets as;
    as.scenario = blob();
    as.leftAgents = r.get<int32_t>();
    as.rightAgents = r.get<int32_t>();
    const int nv = r.get<int32_t>();
    if (nv != 4) throw std::runtime_error("asset bundle: expected 4 variants");
    const int l = leftAgents == -1 ? as.leftAgents : leftAgents;
    const int rr = rightAgents == -1 ? as.rightAgents : rightAgents;
    const bool setup = l != as.leftAgents || rr != as.rightAgents;
    Codec codec;
    for (int i = 0; i < nv; i++) {
        const int rev = r.get<int32_t>(), par = r.get<int32_t>();
        if ((rev != 0 && rev != 1) || (par != 0 && par != 1)) throw std::runtime_error("asset bundle: bad variant");
        AssetVariant &v = as.variants[rev * 2 + par];
        v.reverse = rev;
        v.parity = par;
        v.staticData = parse_static(blob());
        v.world.reset(new Match);
        if (!codec.load_frame(blob(), *v.world)) throw std::runtime_error("asset bundle: bad reset state");
        v.freeControllerCount = codec.freeControllerCount;
        if (setup) {
            setup_agents(*v.world, v.staticData, l, rr, path);
            v.freeControllerCount = v.world->m.freeControllerCount;
        }
        v.scenario = save_scenario(*v.world);
        v.skeletons = parse_skeletons(blob());
        if ((int)v.skeletons.size() != v.staticData.count)
            throw std::runtime_error("asset bundle: expected " + std::to_string(v.staticData.count) +
                                     " skeletons, found " + std::to_string(v.skeletons.size()));
    }
    for (const AssetVariant &v : as.variants)
        if (!v.world) throw std::runtime_error("asset bundle: missing variant");
    as.leftAgents = l;
    as.rightAgents = rr;
    return as;
}

}  // namespace host
}  // namespace cb

# Test-infrastructure shim for the golden-vector generator only: lets the installed antlr4
# 4.13 runtime load the version-3 ATNs that the reference's ANTLR 4.9.2-generated lexer and
# parser carry (constraintflow/ast_cflow/dslLexer.py, dslParser.py).  Importing it replaces
# antlr4.ATNDeserializer before the reference's parser modules are imported.
import antlr4
from antlr4.atn.ATNDeserializer import ATNDeserializer as _D
from antlr4.atn.ATNType import ATNType
from antlr4.Token import Token
from antlr4.IntervalSet import IntervalSet
from antlr4.atn.ATNState import RuleStopState

class V3Deserializer(_D):
    def deserialize(self, data):
        if not isinstance(data, str):
            return super().deserialize(data)
        temp = [ord(c) - 2 for c in data]
        temp[0] = ord(data[0])
        self.data = temp; self.pos = 0
        assert self.readInt() == 3
        for _ in range(8): self.readInt()   # UUID
        atn = self.readATN()
        self.readStates(atn)
        self.readRulesV3(atn)
        self.readModes(atn)
        sets = []
        self.readSetsV3(atn, sets, self.readInt)
        self.readSetsV3(atn, sets, self.readInt32)
        self.readEdges(atn, sets)
        self.readDecisions(atn)
        if atn.grammarType == ATNType.LEXER:
            count = self.readInt()
            atn.lexerActions = [None]*count
            for i in range(count):
                t = self.readInt(); d1 = self.readInt(); d2 = self.readInt()
                if d1 == 0xFFFF: d1 = -1
                if d2 == 0xFFFF: d2 = -1
                atn.lexerActions[i] = self.lexerActionFactory(t, d1, d2)
        self.markPrecedenceDecisions(atn)
        self.verifyATN(atn)
        return atn
    def readInt32(self):
        lo = self.readInt(); hi = self.readInt()
        return lo | (hi << 16)
    def readRulesV3(self, atn):
        nrules = self.readInt()
        if atn.grammarType == ATNType.LEXER:
            atn.ruleToTokenType = [0]*nrules
        atn.ruleToStartState = [0]*nrules
        for i in range(nrules):
            s = self.readInt()
            atn.ruleToStartState[i] = atn.states[s]
            if atn.grammarType == ATNType.LEXER:
                t = self.readInt()
                if t == 0xFFFF: t = Token.EOF
                atn.ruleToTokenType[i] = t
        atn.ruleToStopState = [0]*nrules
        for st in atn.states:
            if isinstance(st, RuleStopState):
                atn.ruleToStopState[st.ruleIndex] = st
                atn.ruleToStartState[st.ruleIndex].stopState = st
    def readSetsV3(self, atn, sets, readUnicode):
        m = self.readInt()
        for _ in range(m):
            iset = IntervalSet(); sets.append(iset)
            n = self.readInt()
            if self.readInt() != 0: iset.addOne(-1)
            for _ in range(n):
                i1 = readUnicode(); i2 = readUnicode()
                iset.addRange(range(i1, i2+1))

antlr4.ATNDeserializer = V3Deserializer
